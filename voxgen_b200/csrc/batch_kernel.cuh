// The batched decode-step kernel: one persistent launch advances up to 16
// "columns" by one token each and reads every weight byte once for all of
// them. A column is a decode position of a stream: one position each of up to
// 16 independent streams (vg_decode_batch), or up to 16
// consecutive positions of one stream (vg_prefill_tokens). The layer sequence
// is record_transformer's (src/baselm.rs:892-1052), as in the single-stream
// step kernel (step_kernel.cuh), whose grid barriers, producer warp and ring
// this kernel shares.
//
// Matvec phases are split over the grid in two dimensions. For each matrix
// kind the host picks C column groups and R = grid / C row groups; CTA
// (r, c) owns the tiles of row group r and the segments of column group c.
// It builds the operand of its K-slice only (S columns x Kc elements), so the
// activation that every CTA would otherwise read whole from L2 is read once
// per row group, and it writes fp32 partial sums for its tiles. After the C
// CTAs of a row group have arrived on their counter, each reduces a share of
// the group's tiles in a fixed order and runs the epilogue (RoPE + fp16 KV
// store, residual add, SwiGLU) for every column.
//
// Operand: each column's slice is scaled by a power of two 2^-e (max below
// 2^14) and split into fp16 hi + lo, so every element keeps 22 significant
// bits whatever the other elements' magnitudes. The weights are the A operand
// of mma.sync m16n8k16 (f16, fp32 accumulation): F16 tiles as stored, Q8_0
// quants converted to fp16 in registers (exact for |q| <= 128). The 16
// columns are two n8 tiles; hi and lo accumulate into one accumulator, and a
// Q8_0 K-step's sum is scaled by the fp16 block scale of each row in fp32.
//
// Attention runs per column: split-K units (column, KV head, 64 positions)
// over the column's own cache, then one merge slice per (column, query head).
// Rows a column reads that this same launch writes (the column's own row, and
// for a prefill run the rows of the earlier columns) are loaded from L2 after
// the barrier; older rows stream through the ring.
#pragma once
#include "step_kernel.cuh"

namespace vg {

constexpr uint32_t kBatchMaxCols = 16;
constexpr uint32_t kBatchMaxRowGroups = 148;
constexpr uint32_t kBatchKinds = 4;  // matvec kinds: QKV, o_proj, gate/up, down

// One column of a batched step. The position is ctrl[kCtrlPos] + off; rows at
// or above ctrl[kCtrlPos] of the column's cache are written by this launch.
struct BatchCol {
  __half *kc, *vc;                 // layer-0 K and V caches of the stream, [kv_head][ctx][head_dim]
  unsigned long long layer_elems;  // elements from one layer's cache to the next
  uint32_t *ctrl;                  // the stream's control block (position; error flag)
  float *out;                      // the stream's final hidden state (written by its last column)
  uint32_t ctx;                    // the stream's cache capacity in positions
  uint32_t off;                    // position of the column within its stream's run
  uint32_t adv;                    // last column of a stream: the run length (position advance); else 0
  uint32_t token;                  // input token id
};

// Split of one matvec kind over the grid: C column groups x R row groups.
struct BatchSplit {
  uint32_t C, R;
};

struct BatchParams {
  const StepLayer *layers;  // [n_layers] (kc/vc unused: caches come from the columns)
  uint32_t n_layers;
  TileGeom g[kBatchKinds];  // QKV, o_proj, gate/up, down
  BatchSplit split[kBatchKinds];
  TileGeom g_tok;
  const uint8_t *tok;       // token table (segmented tiles)
  const float *out_norm;
  const BatchCol *cols;     // [S]
  uint32_t S;
  float *hid_a, *hid_b, *q, *attn;  // [S][H]
  float *gate;                      // [S][F]
  float *part;              // matvec partials [C][part_tiles][16 rows][16 columns]
  uint32_t part_tiles;
  float *ssb;               // partial sums of squares [R][C][16]
  float *apart;             // attention partials [S][kv_heads][max_chunks][G][head_dim]
  float2 *apart_ml;         // their (max, sum) [S][kv_heads][max_chunks][G]
  unsigned long long *ready;  // [S][kv_heads] unit arrivals, monotonic
  unsigned long long *rgc;    // [kBatchKinds][kBatchMaxRowGroups] row-group arrivals, monotonic
  unsigned long long *bar;    // grid-barrier arrivals
  uint32_t *ctrl;             // the launch's control block (error flag, wait limit)
  const float *inv_freq, *ext;
  float rope_scaling, eps, res_scale, emb_scale, attn_scale;
  uint32_t H, F, heads, kv_heads, head_dim;
  uint32_t chunk, max_chunks;  // attention positions per unit; partial slots per (column, KV head)
  uint32_t merge_dw;           // dimensions of a merge slice (batch_merge_width)
  // shared-memory plan (BatchSmem)
  uint32_t nst, slot, aux_bytes;
};

// Shared memory of a batched-step CTA: the ring and its barriers, two staging
// barriers, the aux region (matvec operand planes + staged input + norm
// weight + per-column scalars, or the attention scratch), a small scratch
// (unit-arrival bases) and the layer table.
struct BatchSmem {
  uint32_t ring, bars, sbar, aux, scr, layers, total;
  __host__ __device__ BatchSmem(const BatchParams &p) {
    ring = 0;
    bars = ring + p.nst * p.slot;
    sbar = bars + p.nst * 16u;
    aux = (sbar + 16u + 127u) & ~127u;
    scr = aux + ((p.aux_bytes + 127u) & ~127u);
    layers = scr + 4096u;
    total = layers + p.n_layers * (uint32_t)sizeof(StepLayer);
  }
};

// Bytes of the warps' partial sums of one group of 4 tiles: [warp][tile][16 rows][16 columns].
constexpr uint32_t kBatchRedBytes = kMvConsumers * 4u * 256u * 4u;

// Matvec operand region of the aux area for a K-slice of kc elements:
// hi plane, lo plane (each 16 columns x kc fp16), the staged fp32 input
// [16][kc] (after the prologue the same bytes hold the warps' partial sums,
// so the region is at least kBatchRedBytes), the staged norm weight [kc],
// then per column 2^e and the sum of squares of the slice.
struct BatchOperand {
  uint32_t hi, lo, stg, red, stw, colv, total;
  __host__ __device__ BatchOperand(uint32_t kc) {
    hi = 0;
    lo = hi + kc * kBatchMaxCols * 2u;
    stg = lo + kc * kBatchMaxCols * 2u;
    red = stg;
    const uint32_t sb = kc * kBatchMaxCols * 4u;
    stw = stg + (sb > kBatchRedBytes ? sb : kBatchRedBytes);
    colv = stw + kc * 4u;
    total = colv + 2u * kBatchMaxCols * 4u;
  }
};

// Byte offset, inside a plane, of operand element k (0 <= k < kc) of column n.
// Q8_0 (K-steps of 32): lane tq of an MMA reads, for K-step kk and column n,
// 16 bytes holding elements 4tq..4tq+3 and 16+4tq..16+4tq+3 (the B fragments
// of the two k16 MMAs of the K-step, in the k order the int8 A fragment
// converts to). F16 (K-steps of 16): 8 bytes holding 2tq, 2tq+1, 8+2tq, 9+2tq.
__host__ __device__ inline uint32_t batch_bfrag_off(bool q8, uint32_t k, uint32_t n) {
  if (q8) {
    const uint32_t kk = k >> 5, w = k & 31u;
    return ((kk * kBatchMaxCols + n) * 4u + ((w & 15u) >> 2)) * 16u + (w >> 4) * 8u + (w & 3u) * 2u;
  }
  const uint32_t kk = k >> 4, w = k & 15u;
  return ((kk * kBatchMaxCols + n) * 4u + ((w & 7u) >> 1)) * 8u + (w >> 3) * 4u + (w & 1u) * 2u;
}

// int8x4 -> two fp16x2 (elements 0,1 and 2,3), exactly: (q ^ 0x80) is q + 128,
// and the fp16 with bits 0x6400 | u is 1024 + u, so subtracting 1152 gives q.
__device__ __forceinline__ void i8x4_to_h2x2(uint32_t a, uint32_t &lo, uint32_t &hi) {
  const uint32_t x = a ^ 0x80808080u;
  const uint32_t l = __byte_perm(x, 0x64646464u, 0x4140u), h = __byte_perm(x, 0x64646464u, 0x4342u);
  const __half2 bias = __halves2half2(__ushort_as_half(0x6480u), __ushort_as_half(0x6480u));  // 1152
  const __half2 rl = __hsub2(*reinterpret_cast<const __half2 *>(&l), bias);
  const __half2 rh = __hsub2(*reinterpret_cast<const __half2 *>(&h), bias);
  lo = *reinterpret_cast<const uint32_t *>(&rl);
  hi = *reinterpret_cast<const uint32_t *>(&rh);
}

// D = A * B + 0 (f16, fp32 accumulation): the first MMA of a block sum.
__device__ __forceinline__ void mma_f16_zero(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%10, %10, %10, %10};"
      : "=f"(c[0]), "=f"(c[1]), "=f"(c[2]), "=f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "f"(0.0f));
}

// Activation operand of a batched matvec over the K-slice [k0, k0 + kc) of
// an input of `ld` floats per column: the consumer warps (256 threads) take
// one column per half-warp. The input slice of every column is in stg (fp32
// [16][kc]) and, with rms, the norm weight slice in stw. With rms the operand
// is x * w (RMSNorm deferred to the output rows) and the slice's sum of
// squares of x goes to colv[16 + n]; colv[n] receives 2^e. Columns >= S are
// zero.
template <bool Q8>
__device__ __forceinline__ void batch_activation(const BatchOperand &O, uint8_t *aux, uint32_t kc, uint32_t S,
                                                 bool rms, uint32_t tid) {
  const uint32_t n = tid >> 4, t16 = tid & 15u;  // column, thread within the half-warp
  const float *stg = reinterpret_cast<const float *>(aux + O.stg) + n * kc;
  const float *stw = reinterpret_cast<const float *>(aux + O.stw);
  float *colv = reinterpret_cast<float *>(aux + O.colv);
  uint8_t *hi = aux + O.hi, *lo = aux + O.lo;
  const bool live = n < S;
  float m = 0.f, ss = 0.f;
  if (live) {
#pragma unroll 1
    for (uint32_t k = t16 * 4u; k < kc; k += 64u) {
      float4 v = *reinterpret_cast<const float4 *>(stg + k);
      ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
      if (rms) {
        const float4 w = *reinterpret_cast<const float4 *>(stw + k);
        v.x = __fmul_rn(v.x, w.x);
        v.y = __fmul_rn(v.y, w.y);
        v.z = __fmul_rn(v.z, w.z);
        v.w = __fmul_rn(v.w, w.w);
      }
      m = fmaxf(m, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
    }
  }
  // half-warp reductions (xor offsets below 16 stay inside the half)
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) {
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    ss += __shfl_xor_sync(0xffffffffu, ss, o);
  }
  const uint32_t ef = (__float_as_uint(m) >> 23) & 0xFFu;
  const int e = ef < 20 ? 0 : (int)ef - 127 - 13;  // max |x| 2^-e < 2^14
  const float inv = pow2f(-e);
  if (t16 == 0) {
    colv[n] = pow2f(e);
    colv[kBatchMaxCols + n] = ss;
  }
#pragma unroll 1
  for (uint32_t k = t16 * 4u; k < kc; k += 64u) {
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (live) {
      v = *reinterpret_cast<const float4 *>(stg + k);
      if (rms) {
        const float4 w = *reinterpret_cast<const float4 *>(stw + k);
        v.x = __fmul_rn(v.x, w.x);
        v.y = __fmul_rn(v.y, w.y);
        v.z = __fmul_rn(v.z, w.z);
        v.w = __fmul_rn(v.w, w.w);
      }
    }
    const float vv[4] = {v.x * inv, v.y * inv, v.z * inv, v.w * inv};
    __half h[4], l[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      h[i] = __float2half_rn(vv[i]);
      l[i] = __float2half_rn(vv[i] - __half2float(h[i]));
    }
    if (Q8) {  // elements k..k+3 are 4 consecutive halves of one lane's 16 bytes
      const uint32_t o = batch_bfrag_off(true, k, n);
      *reinterpret_cast<uint2 *>(hi + o) = make_uint2(pack_half2(h[0], h[1]), pack_half2(h[2], h[3]));
      *reinterpret_cast<uint2 *>(lo + o) = make_uint2(pack_half2(l[0], l[1]), pack_half2(l[2], l[3]));
    } else {  // two pairs, in the 8-byte words of two lanes
      const uint32_t o0 = batch_bfrag_off(false, k, n), o1 = batch_bfrag_off(false, k + 2u, n);
      *reinterpret_cast<uint32_t *>(hi + o0) = pack_half2(h[0], h[1]);
      *reinterpret_cast<uint32_t *>(lo + o0) = pack_half2(l[0], l[1]);
      *reinterpret_cast<uint32_t *>(hi + o1) = pack_half2(h[2], h[3]);
      *reinterpret_cast<uint32_t *>(lo + o1) = pack_half2(l[2], l[3]);
    }
  }
}


// The share of one matvec kind a CTA owns: tiles [t0, t0 + nt) of row group r
// and segments [s0, s0 + ns) of every such tile (column group c).
struct BatchRun {
  uint32_t t0, nt, s0, ns, r, c;
  bool live;
};
__device__ __forceinline__ BatchRun batch_run(const TileGeom &g, const BatchSplit &sp) {
  BatchRun b{};
  b.live = blockIdx.x < sp.R * sp.C;
  if (!b.live) return b;
  const uint32_t T = g.tiles(), NS = g.nseg();
  b.r = blockIdx.x / sp.C;
  b.c = blockIdx.x - b.r * sp.C;
  b.t0 = T * b.r / sp.R;
  b.nt = T * (b.r + 1u) / sp.R - b.t0;
  b.s0 = NS * b.c / sp.C;
  b.ns = NS * (b.c + 1u) / sp.C - b.s0;
  return b;
}
// Tile groups of a run: groups of 4 consecutive tiles (the last may hold fewer),
// each streamed segment by segment. A stage is one group's tiles at one
// segment, so the phase has groups x ns stages.
__device__ __forceinline__ uint32_t batch_groups(const BatchRun &b) { return (b.nt + 3u) / 4u; }
__device__ __forceinline__ uint32_t batch_stages(const BatchRun &b) { return batch_groups(b) * b.ns; }

// Ring stage k stages after rp: slot and the parity of that use.
__device__ __forceinline__ void ring_at(const RingPos &rp, uint32_t k, uint32_t nst, uint32_t &slot, uint32_t &par) {
  const uint32_t s = rp.slot + k;
  slot = s % nst;
  par = rp.phase ^ ((s / nst) & 1u);
}

// Producer side of a batched matvec: for every group of up to 4 tiles and
// every segment of the slice, one stage holding that segment of each tile of
// the group (one bulk copy per tile).
__device__ __forceinline__ bool batch_produce(const MvRing &R, const uint8_t *w, const TileGeom &g, const BatchRun &b,
                                              RingPos &rp, const uint32_t *abort_flag, uint32_t *err) {
  const uint32_t SEGB = g.seg_bytes(), NS = g.nseg();
  for (uint32_t q = 0; q < batch_groups(b); ++q) {
    const uint32_t nq = min(4u, b.nt - 4u * q);
    for (uint32_t sgi = 0; sgi < b.ns; ++sgi) {
      if (!ring_claim(R, rp, nq * SEGB, abort_flag, err)) return false;
      uint8_t *dst = R.ring + rp.slot * R.slot;
      for (uint32_t j = 0; j < nq; ++j)
        bulk_g2s_stream(dst + j * SEGB, w + ((uint64_t)(b.t0 + 4u * q + j) * NS + b.s0 + sgi) * SEGB, SEGB, &R.full[rp.slot]);
      rp.next(R.nst);
    }
  }
  return true;
}

// Consumer side of a batched matvec. Every warp takes every stage: warp cw
// does K-step cw of the stage's segment for each of its (up to 4) tiles, the
// B fragments loaded once for all of them, and accumulates over the group's
// segments. After a group the warps' sums go to shared memory (red), and the
// CTA adds them in warp order, times each column's 2^e, into
// part[c][tile][row][column].
template <bool Q8>
__device__ __forceinline__ void batch_consume(const MvRing &R, RingPos &rp, const BatchRun &b, const TileGeom &g,
                                              uint8_t *aux, const BatchOperand &O, uint32_t S, float *part,
                                              uint32_t part_tiles, uint32_t cw, uint32_t lane,
                                              const uint32_t *abort_flag, uint32_t *err, bool &ok) {
  constexpr uint32_t NCT = kMvConsumers * 32;
  const uint32_t SEGB = g.seg_bytes(), tid = cw * 32u + lane;
  const uint32_t gq = lane >> 2, tq = lane & 3u;
  const float *colv = reinterpret_cast<const float *>(aux + O.colv);
  const uint8_t *hi = aux + O.hi, *lo = aux + O.lo;
  float *red = reinterpret_cast<float *>(aux + O.red);
  (void)S;  // both n8 tiles are always computed; columns >= S hold zeros
  for (uint32_t q = 0; q < batch_groups(b); ++q) {
    const uint32_t nq = min(4u, b.nt - 4u * q);
    float tot[4][2][4];
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int i = 0; i < 4; ++i) tot[j][nt][i] = 0.f;
#pragma unroll 1
    for (uint32_t sgi = 0; sgi < b.ns; ++sgi) {
      if (!mbar_wait_bounded(&R.full[rp.slot], rp.phase, abort_flag)) {
        set_error(err, kErrConsumerWait);
        ok = false;
      }
      const uint8_t *st = R.ring + rp.slot * R.slot;
      const uint32_t kk = sgi * kSegSteps + cw;  // K-step within the slice
      // the 4 tiles' work is issued in lock-step so their MMA chains overlap; a
      // group of fewer tiles repeats its last tile, whose sums are not kept
      const uint8_t *sg[4];
#pragma unroll
      for (uint32_t j = 0; j < 4; ++j) sg[j] = st + min(j, nq - 1u) * SEGB + cw * kStepBytes;
      if constexpr (Q8) {
        const uint32_t bo = ((kk * kBatchMaxCols + gq) * 4u + tq) * 16u;
        const uint4 bh0 = *reinterpret_cast<const uint4 *>(hi + bo), bl0 = *reinterpret_cast<const uint4 *>(lo + bo);
        const uint4 bh1 = *reinterpret_cast<const uint4 *>(hi + bo + 8u * 64u);
        const uint4 bl1 = *reinterpret_cast<const uint4 *>(lo + bo + 8u * 64u);
        uint32_t a[4][4];
        float2 d[4];
#pragma unroll
        for (uint32_t j = 0; j < 4; ++j) {
          ldmatrix_x4(a[j], sg[j] + lane * 16u);
          d[j] = __half22float2(*reinterpret_cast<const __half2 *>(sg[j] - cw * kStepBytes + kSegQsBytes + gq * 32u + cw * 4u));
        }
        float c[4][2][4];
        uint32_t A[4][4];
        // K columns 0-15 of the step (int8 A fragment registers 0 and 1)
#pragma unroll
        for (uint32_t j = 0; j < 4; ++j) {
          i8x4_to_h2x2(a[j][0], A[j][0], A[j][2]);
          i8x4_to_h2x2(a[j][1], A[j][1], A[j][3]);
        }
#pragma unroll
        for (uint32_t j = 0; j < 4; ++j) {
          mma_f16_zero(c[j][0], A[j], bh0.x, bh0.y);
          mma_f16_zero(c[j][1], A[j], bh1.x, bh1.y);
        }
#pragma unroll
        for (uint32_t j = 0; j < 4; ++j) {
          mma_f16(c[j][0], A[j], bl0.x, bl0.y);
          mma_f16(c[j][1], A[j], bl1.x, bl1.y);
        }
        // K columns 16-31 (registers 2 and 3)
#pragma unroll
        for (uint32_t j = 0; j < 4; ++j) {
          i8x4_to_h2x2(a[j][2], A[j][0], A[j][2]);
          i8x4_to_h2x2(a[j][3], A[j][1], A[j][3]);
        }
#pragma unroll
        for (uint32_t j = 0; j < 4; ++j) {
          mma_f16(c[j][0], A[j], bh0.z, bh0.w);
          mma_f16(c[j][1], A[j], bh1.z, bh1.w);
        }
#pragma unroll
        for (uint32_t j = 0; j < 4; ++j) {
          mma_f16(c[j][0], A[j], bl0.z, bl0.w);
          mma_f16(c[j][1], A[j], bl1.z, bl1.w);
        }
#pragma unroll
        for (uint32_t j = 0; j < 4; ++j)
#pragma unroll
          for (uint32_t nt = 0; nt < 2; ++nt) {
            tot[j][nt][0] = fmaf(c[j][nt][0], d[j].x, tot[j][nt][0]);
            tot[j][nt][1] = fmaf(c[j][nt][1], d[j].x, tot[j][nt][1]);
            tot[j][nt][2] = fmaf(c[j][nt][2], d[j].y, tot[j][nt][2]);
            tot[j][nt][3] = fmaf(c[j][nt][3], d[j].y, tot[j][nt][3]);
          }
      } else {
        const uint32_t bo = ((kk * kBatchMaxCols + gq) * 4u + tq) * 8u;
        const uint2 bh0 = *reinterpret_cast<const uint2 *>(hi + bo), bl0 = *reinterpret_cast<const uint2 *>(lo + bo);
        const uint2 bh1 = *reinterpret_cast<const uint2 *>(hi + bo + 8u * 32u);
        const uint2 bl1 = *reinterpret_cast<const uint2 *>(lo + bo + 8u * 32u);
        uint32_t a[4][4];
#pragma unroll
        for (uint32_t j = 0; j < 4; ++j) ldmatrix_x4(a[j], sg[j] + lane * 16u);
#pragma unroll
        for (uint32_t j = 0; j < 4; ++j) {
          mma_f16(tot[j][0], a[j], bh0.x, bh0.y);
          mma_f16(tot[j][1], a[j], bh1.x, bh1.y);
        }
#pragma unroll
        for (uint32_t j = 0; j < 4; ++j) {
          mma_f16(tot[j][0], a[j], bl0.x, bl0.y);
          mma_f16(tot[j][1], a[j], bl1.x, bl1.y);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&R.empty[rp.slot]);
      rp.next(R.nst);
    }
    // the warps' sums of the group: red[warp][tile][row][column]; lane (gq, tq)
    // holds rows gq, gq + 8 and columns 8 nt + 2 tq, 8 nt + 2 tq + 1
#pragma unroll
    for (uint32_t j = 0; j < 4; ++j) {
      if (j >= nq) break;
      float *rt = red + (cw * 4u + j) * 256u;
#pragma unroll
      for (uint32_t nt = 0; nt < 2; ++nt) {
        const uint32_t col = nt * 8u + 2u * tq;
        *reinterpret_cast<float2 *>(rt + gq * 16u + col) = make_float2(tot[j][nt][0], tot[j][nt][1]);
        *reinterpret_cast<float2 *>(rt + (gq + 8u) * 16u + col) = make_float2(tot[j][nt][2], tot[j][nt][3]);
      }
    }
    named_bar(1, NCT);
    for (uint32_t v = tid; v < nq * 256u; v += NCT) {
      const uint32_t j = v >> 8, e = v & 255u;
      float a = 0.f;
#pragma unroll
      for (uint32_t w = 0; w < kMvConsumers; ++w) a += red[(w * 4u + j) * 256u + e];
      part[((size_t)b.c * part_tiles + b.t0 + 4u * q + j) * 256u + e] = a * colv[e & 15u];
    }
    named_bar(1, NCT);  // red reuse
  }
}

// Reduction of a row group's partials and the epilogue, after the C CTAs of
// the group have arrived: this CTA takes the group's tiles c, c + C, ...; a
// thread takes (tile, row pair p / p + 8, column n) and adds the C partials
// in column-group order. rs[n] is the column's deferred RMSNorm scale (or 1).
template <class Epi>
__device__ __forceinline__ void batch_reduce(const BatchRun &b, uint32_t C, const float *part, uint32_t part_tiles,
                                             const float *rs, uint32_t S, uint32_t tid, Epi epi) {
  const uint32_t half = tid >> 7, pr = (tid >> 4) & 7u, n = tid & 15u;
  const size_t stride = (size_t)part_tiles * 256u;
  // two tiles per iteration, their loads in flight together
  for (uint32_t i = half; b.c + i * C < b.nt; i += 4u) {
    const uint32_t t = b.t0 + b.c + i * C;
    const bool two = b.c + (i + 2u) * C < b.nt;
    const uint32_t t2 = two ? t + 2u * C : t;
    const float *pt = part + (size_t)t * 256u + pr * 16u + n, *pu = part + (size_t)t2 * 256u + pr * 16u + n;
    float a = 0.f, c2 = 0.f, a2 = 0.f, c3 = 0.f;
    for (uint32_t cg = 0; cg < C; ++cg) {
      a += __ldcg(pt + cg * stride);
      c2 += __ldcg(pt + cg * stride + 128u);
      a2 += __ldcg(pu + cg * stride);
      c3 += __ldcg(pu + cg * stride + 128u);
    }
    if (n < S) {
      epi(t * kTileRows + pr, n, a * rs[n], c2 * rs[n]);
      if (two) epi(t2 * kTileRows + pr, n, a2 * rs[n], c3 * rs[n]);
    }
  }
}

enum : uint32_t { kBkQkv = 0, kBkO = 1, kBkGu = 2, kBkDown = 3 };

// Positions of a batched attention unit for head_dim D: 16-row MMA tiles of K
// and V rows that fit one stage slot together (a slot holds 16 KiB or more).
__host__ __device__ constexpr uint32_t batch_chunk(uint32_t D) { return D >= 128u ? 32u : 64u; }

// aux bytes of an attention phase: every warp's P of its unit (hi and lo,
// [8 heads][chunk] fp16), or a merge slice's chunk weights [max_chunks][8]
// followed by [32][8] partial maxima, [32][8] partial sums and the parts'
// outputs (at most 4 floats per thread).
__host__ __device__ inline uint32_t batch_attn_bytes(uint32_t chunk, uint32_t max_chunks) {
  const uint32_t units = kMvConsumers * 2u * 8u * chunk * 2u;
  const uint32_t merge = (max_chunks * 8u + 2u * 256u + kMvConsumers * 32u * 4u) * 4u;
  return units > merge ? units : merge;
}

// Dimensions of a merge slice for S columns: the narrowest of 16, 32, ...,
// head_dim whose (column, KV head, slice) count fits the grid, so each CTA
// merges one slice at most, as long as a slice's threads (width x group / 4
// heads loaded at once) fit the CTA.
__host__ __device__ inline uint32_t batch_merge_width(uint32_t S, uint32_t kv_heads, uint32_t D, uint32_t G,
                                                      uint32_t grid) {
  const uint32_t gv = G % 4u == 0 ? G / 4u : G / 2u;
  uint32_t dw = 16u;
  while (dw < D && 2u * dw * gv <= kMvConsumers * 32u && S * kv_heads * (D / dw) > grid) dw *= 2u;
  return dw;
}

// Attention unit u of a batched step: units are ordered by column, KV head,
// chunk; cu0 holds each column's first unit.
struct BatchUnit {
  uint32_t n, kvh, c, r0, len, staged;
};
__device__ __forceinline__ BatchUnit batch_unit(uint32_t u, const uint32_t *cu0, const uint32_t *cnch,
                                                const uint32_t *cpos, const uint32_t *cff, uint32_t S, uint32_t chunk) {
  BatchUnit a;
  uint32_t n = 0;
  while (n + 1u < S && cu0[n + 1u] <= u) ++n;
  const uint32_t w = u - cu0[n], nch = cnch[n];
  a.n = n;
  a.kvh = w / nch;
  a.c = w - a.kvh * nch;
  a.r0 = a.c * chunk;
  const uint32_t r1 = min(a.r0 + chunk, cpos[n] + 1u);
  a.len = r1 - a.r0;
  const uint32_t f = min(r1, cff[n]);  // rows below f were written by earlier launches
  a.staged = f > a.r0 ? f - a.r0 : 0u;
  return a;
}

// One CTA of kMvThreads (8 consumer warps + the producer warp) per SM.
template <bool Q8, int DPL>
__global__ void __launch_bounds__(kMvThreads, 1) decode_batch_kernel(const __grid_constant__ BatchParams p) {
  constexpr uint32_t NCT = kMvConsumers * 32;
  constexpr uint32_t D = 32u * DPL;
  extern __shared__ __align__(128) uint8_t smem[];
  const BatchSmem L(p);
  MvRing R;
  R.ring = smem + L.ring;
  R.full = reinterpret_cast<uint64_t *>(smem + L.bars);
  R.empty = R.full + p.nst;
  R.nst = p.nst;
  R.slot = p.slot;
  uint8_t *aux = smem + L.aux;
  uint64_t *sbar = reinterpret_cast<uint64_t *>(smem + L.sbar);  // staging: input rows, norm weight
  StepLayer *layers = reinterpret_cast<StepLayer *>(smem + L.layers);
  // scratch: per-column state, row scales, barrier bases, unit-arrival bases
  uint32_t *cpos = reinterpret_cast<uint32_t *>(smem + L.scr);  // [16] position
  uint32_t *cff = cpos + 16;                                     // [16] first row written by this launch
  uint32_t *cnch = cpos + 32;                                    // [16] attention chunks
  uint32_t *cu0 = cpos + 48;                                     // [17] first unit of each column
  float *rsc = reinterpret_cast<float *>(smem + L.scr + 384u);    // [16] deferred RMSNorm scales
  float *red = reinterpret_cast<float *>(smem + L.scr + 448u);    // [16] final-norm reduction
  unsigned long long *sb = reinterpret_cast<unsigned long long *>(smem + L.scr + 512u);  // [1 + 4]
  unsigned long long *srdy = reinterpret_cast<unsigned long long *>(smem + L.scr + 1024u);  // [S * kv_heads]
  BatchCol *scol = reinterpret_cast<BatchCol *>(smem + L.scr + 2048u);  // [16]

  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
  uint32_t *err = p.ctrl + kCtrlErr;
  const uint32_t nb = p.n_layers * kPhasesPerLayer;
  const uint32_t G = p.heads / p.kv_heads, S = p.S;

  if (threadIdx.x == 0) {
    for (uint32_t i = 0; i < R.nst; ++i) {
      mbar_init(&R.full[i], 1);
      mbar_init(&R.empty[i], kMvConsumers);
    }
    mbar_init(&sbar[0], 1);
    mbar_init(&sbar[1], 1);
    fence_mbar_init();
    // every CTA arrives nb times per launch at the grid barrier, and the C
    // CTAs of a row group C times per layer at the group's counter
    const unsigned long long c = ld_acquire_u64(p.bar), unit = (unsigned long long)nb * gridDim.x;
    sb[0] = c - c % unit;
    for (uint32_t k = 0; k < kBatchKinds; ++k) {
      const BatchSplit sp = p.split[k];
      sb[1 + k] = 0;
      if (blockIdx.x < sp.R * sp.C) {
        const unsigned long long v = ld_acquire_u64(p.rgc + k * kBatchMaxRowGroups + blockIdx.x / sp.C);
        sb[1 + k] = v - v % ((unsigned long long)sp.C * p.n_layers);
      }
    }
  }
  for (uint32_t i = threadIdx.x; i < p.n_layers * (uint32_t)sizeof(StepLayer) / 8u; i += blockDim.x)
    reinterpret_cast<unsigned long long *>(layers)[i] = reinterpret_cast<const unsigned long long *>(p.layers)[i];
  for (uint32_t i = threadIdx.x; i < S * (uint32_t)sizeof(BatchCol) / 8u; i += blockDim.x)
    reinterpret_cast<unsigned long long *>(scol)[i] = reinterpret_cast<const unsigned long long *>(p.cols)[i];
  // read before this CTA's first arrival (the first unit release of the
  // launch comes after the first grid barrier)
  for (uint32_t i = threadIdx.x; i < S * p.kv_heads; i += blockDim.x) srdy[i] = ld_acquire_u64(p.ready + i);
  __syncthreads();
  if (threadIdx.x < S) {
    const BatchCol &cl = scol[threadIdx.x];
    const uint32_t f = cl.ctrl[kCtrlPos];
    uint32_t pos = f + cl.off;
    if (pos >= cl.ctx) {
      set_error(err, kErrPosition);
      pos = cl.ctx - 1u;
    }
    cpos[threadIdx.x] = pos;
    cff[threadIdx.x] = min(f, pos);
    cnch[threadIdx.x] = (pos + p.chunk) / p.chunk;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    uint32_t u = 0;
    for (uint32_t n = 0; n < S; ++n) {
      cu0[n] = u;
      u += p.kv_heads * cnch[n];
    }
    cu0[S] = u;
  }
  __syncthreads();
  const unsigned long long base = sb[0];
  const uint32_t n_units = cu0[S];

  // ---------------- producer ----------------
  if (warp == kMvConsumers) {
    if (lane == 0) {
      RingPos rp;
      bool live = true;
      for (uint32_t ph = 0; ph < nb && live; ++ph) {
        const uint32_t l = ph / kPhasesPerLayer, kind = ph - l * kPhasesPerLayer;
        const StepLayer &Ly = layers[l];
        if (kind == kPhAttn) {
          // one stage per unit of this CTA: its cached K rows, then its V rows
          for (uint32_t i = 0; live; ++i) {
            bool more = true;
            for (uint32_t w = 0; w < kMvConsumers && live; ++w) {
              const uint32_t u = (i * gridDim.x + blockIdx.x) * kMvConsumers + w;
              if (u >= n_units) {
                more = false;
                break;
              }
              const BatchUnit a = batch_unit(u, cu0, cnch, cpos, cff, S, p.chunk);
              const BatchCol &cl = scol[a.n];
              const size_t off = (size_t)l * cl.layer_elems + ((size_t)a.kvh * cl.ctx + a.r0) * D;
              const uint32_t bytes = a.staged * D * 2u;
              live = ring_claim(R, rp, 2u * bytes, err, err);
              if (!live) break;
              if (bytes) {
                uint8_t *dst = R.ring + rp.slot * R.slot;
                bulk_g2s_stream(dst, cl.kc + off, bytes, &R.full[rp.slot]);
                bulk_g2s_stream(dst + p.chunk * D * 2u, cl.vc + off, bytes, &R.full[rp.slot]);
              }
              rp.next(R.nst);
            }
            if (!more) break;
          }
          continue;
        }
        const uint32_t k = kind == kPhQkv ? kBkQkv : kind == kPhO ? kBkO : kind == kPhGu ? kBkGu : kBkDown;
        const uint8_t *w = k == kBkQkv ? Ly.qkv : k == kBkO ? Ly.o : k == kBkGu ? Ly.gateup : Ly.down;
        const BatchRun b = batch_run(p.g[k], p.split[k]);
        if (b.live) live = batch_produce(R, w, p.g[k], b, rp, err, err);
      }
      if (live) mv_drain(R, rp, err);
    }
    return;
  }

  // ---------------- consumers ----------------
  const uint32_t cw = warp, tid = cw * 32u + lane;
  RingPos rp;
  bool ok = true;
  uint32_t spar = 0;  // parities of the two staging barriers
  auto wait_phase = [&](uint32_t ph) {
    if (tid == 0 && ph > 0 && !grid_wait(p.bar, base + (unsigned long long)ph * gridDim.x, err))
      set_error(err, kErrGridWait);
    named_bar(1, NCT);
  };
  auto arrive = [&] {
    named_bar(1, NCT);
    if (tid == 0) grid_arrive(p.bar);
  };

  // One matvec phase of kind k at layer l: operand of this CTA's K-slice, K
  // loop, partials, row-group arrival, reduction of its share and epilogue.
  auto matvec = [&](uint32_t k, uint32_t ph, uint32_t l) {
    const StepLayer &Ly = layers[l];
    const TileGeom &g = p.g[k];
    const BatchSplit sp = p.split[k];
    const BatchRun b = batch_run(g, sp);
    const uint32_t kc = b.ns * g.seg_cols(), k0 = b.s0 * g.seg_cols();
    const BatchOperand O(kc);
    const bool rms = k == kBkQkv || k == kBkGu;
    const bool tokin = k == kBkQkv && l == 0;  // layer 0 reads the token rows
    const float *src = k == kBkQkv ? p.hid_a : k == kBkO ? p.attn : k == kBkGu ? p.hid_b : p.gate;
    const uint32_t ld = k == kBkDown ? p.F : p.H;
    const uint32_t cols = g.cols;
    // the slice's columns inside the input (the last group may reach into the
    // matrix's zero padding, where the staged input must be zero as well)
    const uint32_t valid = b.live ? min(kc, cols - k0) : 0u;
    // the norm weight does not depend on the step: copied before the wait
    if (b.live && rms && tid == 0) {
      mbar_arrive_expect_tx(sbar + 1, valid * 4u);
      bulk_g2s(aux + O.stw, (k == kBkQkv ? Ly.attn_norm : Ly.ffn_norm) + k0, valid * 4u, sbar + 1);
    }
    if (tid == 0) {
      if (ph > 0 && !grid_wait(p.bar, base + (unsigned long long)ph * gridDim.x, err)) set_error(err, kErrGridWait);
      if (b.live && !tokin) {
        fence_proxy_async_global();
        mbar_arrive_expect_tx(sbar, S * valid * 4u);
        for (uint32_t n = 0; n < S; ++n)
          bulk_g2s(aux + O.stg + n * kc * 4u, src + (size_t)n * ld + k0, valid * 4u, sbar);
      }
    }
    if (b.live && valid < kc) {  // the padding part of the slice: zero input and weight
      float *stg = reinterpret_cast<float *>(aux + O.stg), *stw = reinterpret_cast<float *>(aux + O.stw);
      const uint32_t pad = kc - valid;
      for (uint32_t i = tid; i < S * pad; i += NCT) stg[(i / pad) * kc + valid + i % pad] = 0.f;
      for (uint32_t i = tid; i < pad; i += NCT) stw[valid + i] = 0.f;
    }
    named_bar(1, NCT);
    if (b.live) {
      float *stg = reinterpret_cast<float *>(aux + O.stg);
      if (tokin) {
        // embedding.comp:28-47 for every column; row group 0 also stores the
        // rows as the residual stream
        XSrc ts{};
        ts.tab = p.tok;
        ts.g = p.g_tok;
        ts.alpha = p.emb_scale;
        for (uint32_t i = tid; i < S * valid; i += NCT) {
          const uint32_t n = i / valid, kk = i - n * valid;
          ts.token = scol[n].token;
          const float v = xsrc_elem<true>(ts, k0 + kk);
          stg[n * kc + kk] = v;
          if (b.r == 0) p.hid_a[(size_t)n * p.H + k0 + kk] = v;
        }
        named_bar(1, NCT);
      } else {
        if (!mbar_wait_bounded(sbar, spar & 1u, err)) {
          set_error(err, kErrConsumerWait);
          ok = false;
        }
        spar ^= 1u;
      }
      if (rms) {
        if (!mbar_wait_bounded(sbar + 1, (spar >> 1) & 1u, err)) {
          set_error(err, kErrConsumerWait);
          ok = false;
        }
        spar ^= 2u;
      }
      batch_activation<Q8>(O, aux, kc, S, rms, tid);
      named_bar(1, NCT);
      if (tid < kBatchMaxCols) p.ssb[(b.r * sp.C + b.c) * kBatchMaxCols + tid] =
          reinterpret_cast<const float *>(aux + O.colv)[kBatchMaxCols + tid];
      batch_consume<Q8>(R, rp, b, g, aux, O, S, p.part, p.part_tiles, cw, lane, err, err, ok);
      // every partial (and the slice's sums of squares) of the CTA is written:
      // one arrival at the row group
      named_bar(1, NCT);
      if (tid == 0) grid_arrive(p.rgc + k * kBatchMaxRowGroups + b.r);
    }
    if (!b.live) return;
    // wait for the C CTAs of the row group, then reduce this CTA's share
    if (tid == 0 && !grid_wait(p.rgc + k * kBatchMaxRowGroups + b.r,
                               sb[1 + k] + (unsigned long long)sp.C * (l + 1u), err))
      set_error(err, kErrGridWait);
    named_bar(1, NCT);
    if (tid < kBatchMaxCols) {
      float r = 1.0f;
      if (rms) {
        float ss = 0.f;
        for (uint32_t cg = 0; cg < sp.C; ++cg) ss += __ldcg(p.ssb + (b.r * sp.C + cg) * kBatchMaxCols + tid);
        r = 1.0f / sqrtf(ss / (float)cols + p.eps);  // rmsnorm.comp:21-42, deferred to the rows
      }
      rsc[tid] = r;
    }
    named_bar(1, NCT);
    batch_reduce(b, sp.C, p.part, p.part_tiles, rsc, S, tid, [&](uint32_t R0, uint32_t n, float a, float c2) {
      const uint32_t R1 = R0 + 8u;
      if (k == kBkQkv) {
        // QKV: RoPE on the (i, i + d/2) pair in rows R0 / R1, fp16 K and V rows
        // (rope.comp:22-51, store_kv.comp:16-24)
        if (R0 >= g.rows) return;
        const uint32_t H = p.H, KV = p.kv_heads * D, hd = D / 2u, pos = cpos[n];
        const BatchCol &cl = scol[n];
        if (R0 < H + KV) {
          const bool isq = R0 < H;
          const uint32_t Rr = isq ? R0 : R0 - H;
          const uint32_t head = Rr / D, wr = Rr % D, i = (wr / kTileRows) * 8u + (wr % kTileRows);
          rope_pair(a, c2, pos, i, p.inv_freq, p.ext, p.rope_scaling);
          if (isq) {
            p.q[(size_t)n * H + head * D + i] = a;
            p.q[(size_t)n * H + head * D + i + hd] = c2;
          } else {
            __half *dst = cl.kc + (size_t)l * cl.layer_elems + ((size_t)head * cl.ctx + pos) * D;
            dst[kv_swz(pos, i, D)] = __float2half_rn(a);
            dst[kv_swz(pos, i + hd, D)] = __float2half_rn(c2);
          }
        } else {
          const uint32_t v = R0 - H - KV, kvh = v / D, j = v % D;
          __half *dst = cl.vc + (size_t)l * cl.layer_elems + ((size_t)kvh * cl.ctx + pos) * D;
          dst[kv_swz(pos, j, D)] = __float2half_rn(a);
          dst[kv_swz(pos, j + 8u, D)] = __float2half_rn(c2);
        }
      } else if (k == kBkGu) {
        // matvec_swiglu.comp:67: gate row t * 8 + p (rows R0 / R1 hold gate / up)
        const uint32_t o = (R0 / kTileRows) * 8u + (R0 % kTileRows);
        if (2u * o < g.rows)
          p.gate[(size_t)n * p.F + o] = __fmul_rn(__fdiv_rn(a, __fadd_rn(1.0f, expf(-a))), c2);
      } else {
        // residual_rmsnorm.comp:27: hidden + scale * branch
        float *out = k == kBkO ? p.hid_b : p.hid_a;
        const float *res = k == kBkO ? p.hid_a : p.hid_b;
        const size_t rb = (size_t)n * p.H;
        if (R0 < g.rows) out[rb + R0] = __fadd_rn(__ldcg(res + rb + R0), __fmul_rn(a, p.res_scale));
        if (R1 < g.rows) out[rb + R1] = __fadd_rn(__ldcg(res + rb + R1), __fmul_rn(c2, p.res_scale));
      }
    });
  };

  // One attention phase at layer l (attn_scores / softmax / attn_values,
  // split-K). A unit (column, KV head, chunk of p.chunk positions) is one
  // ring stage (its cached K rows, then its V rows) and belongs to one warp,
  // which runs scores, the chunk softmax and the values on the tensor cores
  // and writes the unit's (o, max, sum) partial: the 8 warps of a CTA work on
  // 8 units at once. Unit u goes to CTA (u / 8) % grid, warp u % 8. Then the
  // merge slices, one per (column, KV head, 16 dimensions).
  auto attention = [&](uint32_t ph, uint32_t l) {
    wait_phase(ph);
    constexpr uint32_t KS = D / 16u;  // K-steps of a head row, and 16-dimension blocks
    constexpr uint32_t W2 = D / 2u;   // 32-bit words of a row
    constexpr uint32_t CH = batch_chunk(D), NPT = CH / 16u;  // positions of a unit, 16-row tiles
    const uint32_t gq = lane >> 2, tq = lane & 3u;
    __half *psh = reinterpret_cast<__half *>(aux) + cw * (2u * 8u * CH);  // P of the warp's unit: [8 heads][CH]
    __half *psl = psh + 8u * CH;                                          // its lo halves
    for (uint32_t i = 0;; ++i) {
      bool more = true;
      for (uint32_t w = 0; w < kMvConsumers; ++w) {
        const uint32_t u = (i * gridDim.x + blockIdx.x) * kMvConsumers + w;
        if (u >= n_units) {
          more = false;
          break;
        }
        if (!mbar_wait_bounded(&R.full[rp.slot], rp.phase, err)) {
          set_error(err, kErrConsumerWait);
          ok = false;
        }
        if (w == cw) {
          const BatchUnit a = batch_unit(u, cu0, cnch, cpos, cff, S, CH);
          const BatchCol &cl = scol[a.n];
          const size_t lo = (size_t)l * cl.layer_elems + (size_t)a.kvh * cl.ctx * D;
          __half *kS = reinterpret_cast<__half *>(R.ring + rp.slot * R.slot), *vS = kS + CH * D;
          // rows this launch wrote (positions >= cff) come from L2
          const uint32_t fr = a.r0 + a.staged, nfw = (a.len - a.staged) * W2;
          const unsigned int *kg = reinterpret_cast<const unsigned int *>(cl.kc + lo + (size_t)fr * D);
          const unsigned int *vg = reinterpret_cast<const unsigned int *>(cl.vc + lo + (size_t)fr * D);
          for (uint32_t e = lane; e < nfw; e += 32u) {
            reinterpret_cast<uint32_t *>(kS + a.staged * D)[e] = __ldcg(kg + e);
            reinterpret_cast<uint32_t *>(vS + a.staged * D)[e] = __ldcg(vg + e);
          }
          // V rows past the unit's end meet zero weights; make them zero too (all
          // NPT tiles are computed, the scores of rows past the end are masked)
          for (uint32_t e = a.len * W2 + lane; e < CH * W2; e += 32u) reinterpret_cast<uint32_t *>(vS)[e] = 0u;
          // q of head gq of the group as B fragments (rows 2tq, 2tq+1 | 2tq+8, 2tq+9
          // of each K-step), split into fp16 hi + lo; heads >= G are zero
          uint32_t qh[KS][2], ql[KS][2];
          const float *qg = p.q + (size_t)a.n * p.H + ((size_t)a.kvh * G + (gq < G ? gq : 0u)) * D + 2u * tq;
#pragma unroll
          for (uint32_t ks = 0; ks < KS; ++ks) {
            float v[4] = {0.f, 0.f, 0.f, 0.f};
            if (gq < G) {
              const float2 x = __ldcg(reinterpret_cast<const float2 *>(qg + ks * 16u));
              const float2 y = __ldcg(reinterpret_cast<const float2 *>(qg + ks * 16u + 8u));
              v[0] = x.x;
              v[1] = x.y;
              v[2] = y.x;
              v[3] = y.y;
            }
#pragma unroll
            for (int j = 0; j < 2; ++j) {
              const __half h0 = __float2half_rn(v[2 * j]), h1 = __float2half_rn(v[2 * j + 1]);
              qh[ks][j] = pack_half2(h0, h1);
              ql[ks][j] = pack_half2(__float2half_rn(v[2 * j] - __half2float(h0)),
                                     __float2half_rn(v[2 * j + 1] - __half2float(h1)));
            }
          }
          __syncwarp();
          // scores (attn_scores.comp:27-44): S[t][g] = K[t] . q[g] * scale, 16 positions
          // per MMA tile, the tiles' chains interleaved
          float sc[NPT][4];
          float m0 = -INFINITY, m1 = -INFINITY;
          {
            float c[NPT][4], c2[NPT][4];
#pragma unroll
            for (uint32_t pt = 0; pt < NPT; ++pt)
#pragma unroll
              for (int j = 0; j < 4; ++j) c[pt][j] = c2[pt][j] = 0.f;
#pragma unroll
            for (uint32_t ks = 0; ks < KS; ++ks)
#pragma unroll
              for (uint32_t pt = 0; pt < NPT; ++pt) {
                const uint32_t kt = pt * 16u + (lane & 15u);  // this lane's K row (chunk-permuted, kv_swz)
                uint32_t af[4];
                ldmatrix_x4(af, kS + kt * D + kv_swz(a.r0 + kt, (lane >> 4) * 8u + ks * 16u, D));
                mma_f16(c[pt], af, qh[ks][0], qh[ks][1]);
                mma_f16(c2[pt], af, ql[ks][0], ql[ks][1]);
              }
#pragma unroll
            for (uint32_t pt = 0; pt < NPT; ++pt) {
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                const uint32_t t = pt * 16u + gq + (j >> 1) * 8u;
                sc[pt][j] = t < a.len ? __fmul_rn(__fadd_rn(c[pt][j], c2[pt][j]), p.attn_scale) : -INFINITY;
              }
              m0 = fmaxf(m0, fmaxf(sc[pt][0], sc[pt][2]));
              m1 = fmaxf(m1, fmaxf(sc[pt][1], sc[pt][3]));
            }
          }
          // chunk softmax (softmax.comp) of heads 2tq and 2tq + 1 over the positions
          // of the 8 lanes that share tq
#pragma unroll
          for (int o = 4; o < 32; o <<= 1) {
            m0 = fmaxf(m0, __shfl_xor_sync(0xffffffffu, m0, o));
            m1 = fmaxf(m1, __shfl_xor_sync(0xffffffffu, m1, o));
          }
          float l0 = 0.f, l1 = 0.f;
#pragma unroll
          for (uint32_t pt = 0; pt < NPT; ++pt) {
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const float e = sc[pt][j] == -INFINITY ? 0.f : expf(sc[pt][j] - ((j & 1) ? m1 : m0));
              if (j & 1) l1 += e; else l0 += e;
              const uint32_t t = pt * 16u + gq + (j >> 1) * 8u, g = 2u * tq + (j & 1);
              const __half h = __float2half_rn(e);
              psh[g * CH + t] = g < G ? h : __float2half_rn(0.f);
              psl[g * CH + t] = g < G ? __float2half_rn(e - __half2float(h)) : __float2half_rn(0.f);
            }
          }
#pragma unroll
          for (int o = 4; o < 32; o <<= 1) {
            l0 += __shfl_xor_sync(0xffffffffu, l0, o);
            l1 += __shfl_xor_sync(0xffffffffu, l1, o);
          }
          __syncwarp();
          // values (attn_values.comp): O[d][g] = sum_t V[t][d] P[t][g] as (V^T)(P^T)
          const size_t pslot = ((size_t)a.n * p.kv_heads + a.kvh) * p.max_chunks + a.c;
          float *po = p.apart + pslot * D * G;
          const uint32_t vt = ((lane >> 4) & 1u) * 8u + (lane & 7u);  // this lane's V row in each 16 (kv_swz)
          uint32_t pbh[NPT][2], pbl[NPT][2];  // P^T B fragments, the same for every dimension tile
#pragma unroll
          for (uint32_t kk = 0; kk < NPT; ++kk) {
            const uint32_t pb = gq * CH + kk * 16u + 2u * tq;
            pbh[kk][0] = *reinterpret_cast<const uint32_t *>(psh + pb);
            pbh[kk][1] = *reinterpret_cast<const uint32_t *>(psh + pb + 8u);
            pbl[kk][0] = *reinterpret_cast<const uint32_t *>(psl + pb);
            pbl[kk][1] = *reinterpret_cast<const uint32_t *>(psl + pb + 8u);
          }
#pragma unroll(KS > 8u ? 2 : 4)
          for (uint32_t dt = 0; dt < KS; ++dt) {
            float o[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (uint32_t kk = 0; kk < NPT; ++kk) {
              uint32_t af[4];
              ldmatrix_x4_trans(af, vS + (kk * 16u + vt) * D +
                                        kv_swz(a.r0 + kk * 16u + vt, dt * 16u + ((lane >> 3) & 1u) * 8u, D));
              mma_f16(o, af, pbh[kk][0], pbh[kk][1]);
              mma_f16(o, af, pbl[kk][0], pbl[kk][1]);
            }
            // rows d, d + 8 of heads 2tq, 2tq + 1 (G is even)
            if (2u * tq < G) {
              const uint32_t d = dt * 16u + gq;
              *reinterpret_cast<float2 *>(po + d * G + 2u * tq) = make_float2(o[0], o[1]);
              *reinterpret_cast<float2 *>(po + (d + 8u) * G + 2u * tq) = make_float2(o[2], o[3]);
            }
          }
          if (gq == 0) {
            if (2u * tq < G) p.apart_ml[pslot * G + 2u * tq] = make_float2(m0, l0);
            if (2u * tq + 1u < G) p.apart_ml[pslot * G + 2u * tq + 1u] = make_float2(m1, l1);
          }
          // the unit's partials are written: one arrival at its (column, KV head)
          __syncwarp();
          if (lane == 0) grid_arrive(p.ready + a.n * p.kv_heads + a.kvh);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&R.empty[rp.slot]);
        rp.next(R.nst);
      }
      if (!more) break;
    }
    // merge slices (column n, KV head, dimensions DW db .. DW db + DW - 1, DW =
    // p.merge_dw, chosen per launch so that the slices fit the grid):
    // o = sum_c exp(m_c - M) o_c / sum_c exp(m_c - M) l_c over the unit chunks.
    // Each thread loads its first chunks' outputs before the weights are known,
    // and keeps its (max, sum) pairs in registers for the second pass.
    const uint32_t DW = p.merge_dw, NSL = D / DW;
    // thread (dimension DW db + dl, heads hq*VW .. hq*VW + VW - 1, chunk part cp)
    // loads VW heads of one dimension at once; the parts are added in order
    const uint32_t VW = G % 4u == 0 ? 4u : 2u, GV = G / VW, TPR = DW * GV, NPART = NCT / TPR;
    const uint32_t rr = tid % TPR, cp = tid / TPR, dl = rr / GV, hq = rr % GV;
    const uint32_t g = tid & 7u, part = tid >> 3;  // the (max, sum) pass: 32 parts of the chunks per head
    float *sW = reinterpret_cast<float *>(aux);    // [max_chunks][8] chunk weights
    float *sM = sW + p.max_chunks * 8u;            // [32][8] partial maxima
    float *sS = sM + 256u;                         // [32][8] partial sums
    float *so = sS + 256u;                         // [NPART][DW x G] the parts' outputs
    for (uint32_t m = gridDim.x - 1u - blockIdx.x; m < S * p.kv_heads * NSL; m += gridDim.x) {
      const uint32_t n = m / (p.kv_heads * NSL), rem = m - n * p.kv_heads * NSL, kvh = rem / NSL, db = rem - kvh * NSL;
      const uint32_t nch = cnch[n];
      if (tid == 0 && !grid_wait(p.ready + n * p.kv_heads + kvh,
                                 srdy[n * p.kv_heads + kvh] + (unsigned long long)(l + 1u) * nch, err))
        set_error(err, kErrGridWait);
      // (the previous slice's last reads of sM / sS / so come before this barrier)
      named_bar(1, NCT);
      const size_t hb = ((size_t)n * p.kv_heads + kvh) * p.max_chunks;
      const float *ob = p.apart + (hb * D + db * DW + dl) * G + hq * VW;
      auto load = [&](uint32_t c) {
        const float *src = ob + (size_t)c * D * G;
        if (VW == 4u) return __ldcg(reinterpret_cast<const float4 *>(src));
        const float2 x = __ldcg(reinterpret_cast<const float2 *>(src));
        return make_float4(x.x, x.y, 0.f, 0.f);
      };
      constexpr uint32_t MR = 4u, MLR = 4u;
      float4 v[MR];
#pragma unroll
      for (uint32_t i = 0; i < MR; ++i) {
        const uint32_t c = cp + i * NPART;
        v[i] = cp < NPART && c < nch ? load(c) : make_float4(0.f, 0.f, 0.f, 0.f);
      }
      float2 ml[MLR];
      float M = -INFINITY;
#pragma unroll
      for (uint32_t i = 0; i < MLR; ++i) {
        const uint32_t c = part + 32u * i;
        ml[i] = g < G && c < nch ? __ldcg(&p.apart_ml[(hb + c) * G + g]) : make_float2(-INFINITY, 0.f);
        M = fmaxf(M, ml[i].x);
      }
      if (g < G)
        for (uint32_t c = part + 32u * MLR; c < nch; c += 32u) M = fmaxf(M, __ldcg(&p.apart_ml[(hb + c) * G + g]).x);
      sM[part * 8u + g] = M;
      named_bar(1, NCT);
      M = -INFINITY;
#pragma unroll 8
      for (uint32_t q2 = 0; q2 < 32u; ++q2) M = fmaxf(M, sM[q2 * 8u + g]);
      float Lp = 0.f;
#pragma unroll
      for (uint32_t i = 0; i < MLR; ++i) {
        const uint32_t c = part + 32u * i;
        if (g < G && c < nch) {
          const float w = ml[i].x == -INFINITY ? 0.f : expf(ml[i].x - M);
          sW[c * 8u + g] = w;
          Lp = fmaf(w, ml[i].y, Lp);
        }
      }
      if (g < G)
        for (uint32_t c = part + 32u * MLR; c < nch; c += 32u) {
          const float2 m2 = __ldcg(&p.apart_ml[(hb + c) * G + g]);
          const float w = m2.x == -INFINITY ? 0.f : expf(m2.x - M);
          sW[c * 8u + g] = w;
          Lp = fmaf(w, m2.y, Lp);
        }
      sS[part * 8u + g] = Lp;
      named_bar(1, NCT);
      if (cp < NPART) {
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
        auto add = [&](uint32_t c, const float4 &x) {
          const float *w = sW + c * 8u + hq * VW;
          acc[0] = fmaf(w[0], x.x, acc[0]);
          acc[1] = fmaf(w[1], x.y, acc[1]);
          if (VW == 4u) {
            acc[2] = fmaf(w[2], x.z, acc[2]);
            acc[3] = fmaf(w[3], x.w, acc[3]);
          }
        };
#pragma unroll
        for (uint32_t i = 0; i < MR; ++i)
          if (cp + i * NPART < nch) add(cp + i * NPART, v[i]);
        uint32_t c = cp + MR * NPART;
        for (; c + 3u * NPART < nch; c += 4u * NPART) {
          const float4 x0 = load(c), x1 = load(c + NPART), x2 = load(c + 2u * NPART), x3 = load(c + 3u * NPART);
          add(c, x0);
          add(c + NPART, x1);
          add(c + 2u * NPART, x2);
          add(c + 3u * NPART, x3);
        }
        for (; c < nch; c += NPART) add(c, load(c));
        for (uint32_t vv = 0; vv < VW; ++vv) so[cp * DW * G + dl * G + hq * VW + vv] = acc[vv];
      }
      named_bar(1, NCT);
      for (uint32_t i = tid; i < DW * G; i += NCT) {
        const uint32_t dd = db * DW + i / G, gd = i % G;
        float L = 0.f, o = 0.f;
        for (uint32_t q2 = 0; q2 < 32u; ++q2) L += sS[q2 * 8u + gd];
        for (uint32_t q2 = 0; q2 < NPART; ++q2) o += so[q2 * DW * G + i];
        p.attn[(size_t)n * p.H + ((size_t)kvh * G + gd) * D + dd] = o * (1.0f / L);
      }
    }
    arrive();
  };

  for (uint32_t ph = 0; ph < nb; ++ph) {
    const uint32_t l = ph / kPhasesPerLayer, kind = ph - l * kPhasesPerLayer;
    if (kind == kPhAttn) {
      attention(ph, l);
      continue;
    }
    matvec(kind == kPhQkv ? kBkQkv : kind == kPhO ? kBkO : kind == kPhGu ? kBkGu : kBkDown, ph, l);
    arrive();
  }

  // final RMSNorm (rmsnorm.comp:21-42 with output_norm) of column blockIdx.x,
  // into its stream's output when it is the stream's last column
  if (blockIdx.x < S) {
    wait_phase(nb);
    const uint32_t n = blockIdx.x;
    const float *h = p.hid_a + (size_t)n * p.H;
    float ss = 0.f;
    for (uint32_t i = tid; i < p.H; i += NCT) {
      const float v = __ldcg(h + i);
      ss += v * v;
    }
    ss = warp_sum(ss);
    if (lane == 0) red[cw] = ss;
    named_bar(1, NCT);
    float tot = 0.f;
#pragma unroll
    for (int w = 0; w < kMvConsumers; ++w) tot += red[w];
    const float inv_rms = 1.0f / sqrtf(tot / (float)p.H + p.eps);
    if (scol[n].adv)
      for (uint32_t i = tid; i < p.H; i += NCT)
        scol[n].out[i] = __fmul_rn(__fmul_rn(__ldcg(h + i), inv_rms), p.out_norm[i]);
  }
  named_bar(1, NCT);
  if (tid == 0) {
    // this CTA's errors go to every stream of the launch
    const uint32_t e = ld_volatile_u32(err);
    if (e)
      for (uint32_t n = 0; n < S; ++n) atomicOr(scol[n].ctrl + kCtrlErr, e);
    // positions advance once every CTA has read them (they all passed the last barrier)
    if (blockIdx.x == 0)
      for (uint32_t n = 0; n < S; ++n)
        if (scol[n].adv) scol[n].ctrl[kCtrlPos] = cff[n] + scol[n].adv;
  }
}
}  // namespace vg
