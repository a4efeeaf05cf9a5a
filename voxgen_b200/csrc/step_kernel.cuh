// The persistent decode-step kernel: one launch per token for the whole
// BaseLM step (record_transformer, src/baselm.rs:892-1052).
//
// One CTA per SM, all resident (cooperative launch). The step is a fixed
// sequence of phases: per layer QKV (+RoPE, fp16 KV store), attention,
// o_proj (+residual), gate/up (+SwiGLU), down (+residual); then the final
// RMSNorm and, when asked, the LM head. A phase may only read what the
// previous phases wrote, so consecutive phases are separated by a grid
// barrier (a monotonically increasing arrival counter in global memory).
//
// The weights do not depend on anything computed in the step, so each CTA's
// producer warp streams its share of every phase's weights (and the cached K/V
// rows its attention units read) into the shared-memory ring in phase order,
// without waiting for the barriers: while the consumer warps wait for a
// phase's input the ring fills with the next phases' weights, and HBM stays
// busy across phase boundaries. The consumer warps run the same matvec and
// attention code as the standalone kernels, in phase order.
//
// Data produced inside the kernel by other CTAs is read with ld.global.cg
// (L2), never through the non-coherent L1.
#pragma once
#include "kernels.cuh"

namespace vg {

struct StepLayer {
  const uint8_t *qkv, *o, *gateup, *down;  // segmented tiles
  const float *attn_norm, *ffn_norm;
  __half *kc, *vc;                          // this layer's caches, [kv_head][ctx][head_dim]
};

struct StepParams {
  const StepLayer *layers;  // [n_layers], copied into shared memory at start
  uint32_t n_layers;
  TileGeom g_qkv, g_o, g_gu, g_down, g_tok, g_head;
  const uint8_t *tok;       // token table (segmented tiles)
  const uint8_t *head;      // LM head (== tok when tied)
  const float *out_norm;
  float *hid_a, *hid_b;     // residual stream ping-pong (the layer input is hid_a)
  float *q, *attn, *gate, *logits, *out;
  float *part;              // attention partial outputs [kv_heads][max_chunks][G][head_dim]
  float2 *part_ml;          // their running max and sum [kv_heads][max_chunks][G]
  // [kv_heads] attention-unit arrivals, monotonic: each unit adds 1 with
  // release semantics once its partials are written, so a KV head's chunks are
  // all written when its count has grown by the chunk count in this layer
  unsigned long long *ready;
  const float *inv_freq, *ext;
  float rope_scaling, eps, res_scale, emb_scale, logit_scale, attn_scale;
  uint32_t H, F, heads, kv_heads, head_dim, ctx;
  uint32_t chunk, max_chunks;  // attention positions per unit; partial slots per KV head
  uint32_t token_input, want_logits;
  uint32_t *ctrl;
  unsigned long long *bar;  // grid barrier arrivals
  // ResidualLM (pre = 3; else 0): three phases before the layers, FSQ in_proj
  // + bias + quantiser into fsq_lat, FSQ out_proj + bias into fuse_in[0, H)
  // (the LM state) and fsq_res, fusion [fuse_in] + bias into hid_a and fused.
  // With fsq_on = 0 (a text-prefix position, fuse_in[0, H) given) the two FSQ
  // phases only keep their grid barriers.
  uint32_t pre, fsq_on;
  TileGeom g_fin, g_fout, g_fuse;
  const uint8_t *w_fin, *w_fout, *w_fuse;
  const float *b_fin, *b_fout, *b_fuse;
  float fsq_scale;
  const float *res_base;    // FSQ input: the BaseLM hidden state
  float *fsq_lat, *fsq_res, *fuse_in, *fused;
  // shared-memory plan (host and device agree through StepSmem)
  uint32_t nst, slot;       // ring stages and bytes per stage slot
  uint32_t a_bytes, plane;  // activation / attention scratch region and digit-plane stride
  uint32_t rb;              // partial-sum tiles (largest per-CTA tile run of any phase)
  uint32_t xcols;           // longest matvec input (columns)
};

// Shared memory of a step CTA: the ring and its barriers (then the two
// staging barriers), the activation operand / attention scratch, the tile
// partial sums, the staged input vector and RMSNorm weight, the layer table
// and a small scratch.
struct StepSmem {
  uint32_t ring, bars, sbar, aux, red, stg, stw, layers, scr, total;
  __host__ __device__ StepSmem(const StepParams &p) {
    ring = 0;
    bars = ring + p.nst * p.slot;
    sbar = bars + p.nst * 16u;
    aux = sbar + 16u;
    red = aux + ((p.a_bytes + 127u) & ~127u);
    stg = red + p.rb * kMvConsumers * kTileRows * 4u;
    stw = stg + ((p.xcols * 4u + 127u) & ~127u);
    layers = stw + ((p.H * 4u + 127u) & ~127u);
    scr = layers + p.n_layers * (uint32_t)sizeof(StepLayer);
    total = scr + 1024u;
  }
};

// Activation operand of a step matvec (mv_activation's arithmetic) from the
// input staged in shared memory (stg, C floats) and, with rms, the staged
// RMSNorm weight (stw): the groups are looped over instead of unrolled, so
// every phase runs one small copy of this code.
template <bool Q8>
__device__ __forceinline__ void step_activation(uint32_t C, uint32_t cols_pad, bool rms, const float *stg,
                                                const float *stw, float eps, uint8_t *areg, uint32_t plane,
                                                float *scr, uint32_t cw, uint32_t lane, float *xout) {
  constexpr uint32_t NCT = kMvConsumers * 32;
  float *sx = reinterpret_cast<float *>(areg + 3u * plane);      // Q8: 2^e of the whole vector
  float *xscale = reinterpret_cast<float *>(areg + 2u * plane);  // F16: 2^e of the whole vector
  // warp cw takes the groups of 128 elements g * 8 + cw, 4 per lane (mv_activation)
  const uint32_t NGRP = (cols_pad / 32u + 3u) / 4u;
  const uint32_t JG = NGRP > cw ? (NGRP - cw + kMvConsumers - 1) / kMvConsumers : 0u;
  auto elem0 = [&](uint32_t g) { return (g * kMvConsumers + cw) * 128u + lane * 4u; };
  auto ld4 = [&](const float *v, uint32_t k0) {
    if (k0 + 3u < C) return *reinterpret_cast<const float4 *>(v + k0);
    float4 r;
    r.x = k0 < C ? v[k0] : 0.f;
    r.y = k0 + 1u < C ? v[k0 + 1u] : 0.f;
    r.z = k0 + 2u < C ? v[k0 + 2u] : 0.f;
    r.w = k0 + 3u < C ? v[k0 + 3u] : 0.f;
    return r;
  };
  // RMSNorm (rmsnorm.comp:21-42) with the 1/rms factor deferred to the rows
  // when there is no xout (mv_activation)
  const bool defer = rms && xout == nullptr;
  float inv_rms = 1.0f;
  // with the factor deferred, the sum of squares and the operand's largest
  // magnitude come from one pass; the operand is then x * w
  float mdef = 0.f, ss = 0.f;
  if (rms) {
#pragma unroll 1
    for (uint32_t g = 0; g < JG; ++g) {
      const float4 v = ld4(stg, elem0(g));
      ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
      if (defer) {
        const float4 w = ld4(stw, elem0(g));
        mdef = fmaxf(mdef, fmaxf(fmaxf(fabsf(__fmul_rn(v.x, w.x)), fabsf(__fmul_rn(v.y, w.y))),
                                 fmaxf(fabsf(__fmul_rn(v.z, w.z)), fabsf(__fmul_rn(v.w, w.w)))));
      }
    }
    // deferred: the warp's sum of squares is reduced after the digits (only
    // the epilogue reads it)
    if (!defer) {
      ss = warp_sum(ss);
      if (lane == 0) scr[cw] = ss;
      named_bar(1, NCT);
      float tot = 0.f;
#pragma unroll
      for (int w = 0; w < kMvConsumers; ++w) tot += scr[w];
      inv_rms = 1.0f / sqrtf(tot / (float)C + eps);
    }
  }
  auto xval = [&](uint32_t k0) {
    float4 v = ld4(stg, k0);
    if (rms) {
      const float4 w = ld4(stw, k0);
      v.x = __fmul_rn(__fmul_rn(v.x, inv_rms), w.x);
      v.y = __fmul_rn(__fmul_rn(v.y, inv_rms), w.y);
      v.z = __fmul_rn(__fmul_rn(v.z, inv_rms), w.z);
      v.w = __fmul_rn(__fmul_rn(v.w, inv_rms), w.w);
    }
    return v;
  };
  auto put_xout = [&](uint32_t k0, const float4 &v) {
    if (!xout) return;
    if (k0 < C) xout[k0] = v.x;
    if (k0 + 1u < C) xout[k0 + 1u] = v.y;
    if (k0 + 2u < C) xout[k0 + 2u] = v.z;
    if (k0 + 3u < C) xout[k0 + 3u] = v.w;
  };
  if constexpr (Q8) {
    // int8 digits and the whole-vector 2^e (mv_activation)
    float m = mdef;
    if (!defer) {
#pragma unroll 1
      for (uint32_t g = 0; g < JG; ++g) {
        const float4 v = xval(elem0(g));
        m = fmaxf(m, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
      }
    }
    m = warp_max(m);
    if (rms && !defer) named_bar(1, NCT);  // scr[] reuse after the RMSNorm reduction
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
#pragma unroll 1
    for (uint32_t g = 0; g < JG; ++g) {
      const uint32_t k0 = elem0(g), b = k0 >> 5;
      const float4 v = xval(k0);
      put_xout(k0, v);
      int q[3][4];
      split(v.x, q[0][0], q[1][0], q[2][0]);
      split(v.y, q[0][1], q[1][1], q[2][1]);
      split(v.z, q[0][2], q[1][2], q[2][2]);
      split(v.w, q[0][3], q[1][3], q[2][3]);
      if (b * 32u < cols_pad) {
        const uint32_t o = b * 32u + bfrag_byte_q8(k0 & 31u);  // 4 consecutive bytes
#pragma unroll
        for (int d = 0; d < 3; ++d) {
          const uint32_t w = __byte_perm(__byte_perm((uint32_t)q[d][0], (uint32_t)q[d][1], 0x0040u),
                                         __byte_perm((uint32_t)q[d][2], (uint32_t)q[d][3], 0x0040u), 0x5410u);
          *reinterpret_cast<uint32_t *>(areg + d * plane + o) = w;
        }
      }
    }
    if (cw == 0 && lane == 0) *sx = nz ? pow2f(e) : 0.f;
    if (defer) {
      ss = warp_sum(ss);
      if (lane == 0) scr[8 + cw] = ss;
    }
    named_bar(1, NCT);
  } else {
    // whole-vector power-of-two scale, then fp16 hi + lo (mv_activation)
    float m = mdef;
    if (!defer) {
#pragma unroll 1
      for (uint32_t g = 0; g < JG; ++g) {
        const float4 v = xval(elem0(g));
        m = fmaxf(m, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
      }
    }
    m = warp_max(m);
    if (rms && !defer) named_bar(1, NCT);  // scr[] reuse after the RMSNorm reduction
    if (lane == 0) scr[cw] = m;
    named_bar(1, NCT);
    float mx = 0.f;
#pragma unroll
    for (int w = 0; w < kMvConsumers; ++w) mx = fmaxf(mx, scr[w]);
    const uint32_t ef = (__float_as_uint(mx) >> 23) & 0xFFu;
    const int e = ef < 20 ? 0 : (int)ef - 127 - 13;  // max|x| * 2^-e < 2^14
    const float inv = pow2f(-e);
    __half *hi = reinterpret_cast<__half *>(areg), *lo = reinterpret_cast<__half *>(areg + plane);
#pragma unroll 1
    for (uint32_t g = 0; g < JG; ++g) {
      const uint32_t k0 = elem0(g);
      const float4 v4 = xval(k0);
      put_xout(k0, v4);
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
    }
    if (cw == 0 && lane == 0) *xscale = pow2f(e);
    if (defer) {
      ss = warp_sum(ss);
      if (lane == 0) scr[8 + cw] = ss;
    }
    named_bar(1, NCT);
  }
}

// Attention scratch inside the aux region: for a unit, the q fragments of one
// KV group, then the scores of a chunk (rows padded by 4 floats); for a merge
// slice, the chunk weights and 1/sum (max_chunks + 4 floats), then the chunk
// groups' partial rows (4 * consumer threads floats).
__host__ __device__ inline uint32_t step_merge_w_bytes(uint32_t max_chunks) {
  return ((max_chunks + 4u) * 4u + 15u) & ~15u;
}
__host__ __device__ inline uint32_t step_attn_bytes(uint32_t G, uint32_t head_dim, uint32_t chunk,
                                                    uint32_t max_chunks) {
  const uint32_t q_frag = (G + 7u) / 8u * (head_dim / 16u) * 2u * 32u * 8u;
  const uint32_t unit = q_frag + G * ((chunk > max_chunks ? chunk : max_chunks) + 4u) * 4u;
  const uint32_t merge = step_merge_w_bytes(max_chunks) + 4u * kMvConsumers * 32u * 4u;
  return unit > merge ? unit : merge;
}

enum : uint32_t { kPhQkv = 0, kPhAttn = 1, kPhO = 2, kPhGu = 3, kPhDown = 4, kPhasesPerLayer = 5 };

__device__ __forceinline__ void tile_run(const TileGeom &g, uint32_t &t0, uint32_t &t1) {
  const uint32_t T = g.tiles();
  t0 = (uint32_t)((uint64_t)blockIdx.x * T / gridDim.x);
  t1 = (uint32_t)((uint64_t)(blockIdx.x + 1) * T / gridDim.x);
}

// Attention unit u of a step: KV head, chunk, first row, rows, and the rows
// below the current position (cached by earlier steps, bulk-copied).
struct AttnUnit {
  uint32_t kvh, c, r0, len, staged;
};
__device__ __forceinline__ AttnUnit attn_unit(const StepParams &p, uint32_t u, uint32_t nch, uint32_t pos) {
  AttnUnit a;
  a.kvh = u / nch;
  a.c = u % nch;
  a.r0 = a.c * p.chunk;
  const uint32_t r1 = min(a.r0 + p.chunk, pos + 1u);
  a.len = r1 - a.r0;
  a.staged = min(r1, pos) - a.r0;
  return a;
}

// One CTA of kMvThreads (9 warps) per SM. Three warps share one SM
// sub-partition's 16K registers, so a thread may use at most 168.
template <bool Q8, int DPL>
__global__ void __launch_bounds__(kMvThreads, 1) decode_step_kernel(const __grid_constant__ StepParams p) {
  constexpr uint32_t NCT = kMvConsumers * 32;
  constexpr uint32_t D = 32u * DPL;
  extern __shared__ __align__(128) uint8_t smem[];
  const StepSmem L(p);
  MvRing R;
  R.ring = smem + L.ring;
  R.full = reinterpret_cast<uint64_t *>(smem + L.bars);
  R.empty = R.full + p.nst;
  R.nst = p.nst;
  R.slot = p.slot;
  uint8_t *aux = smem + L.aux;
  float *red = reinterpret_cast<float *>(smem + L.red);
  StepLayer *layers = reinterpret_cast<StepLayer *>(smem + L.layers);
  uint64_t *sbar = reinterpret_cast<uint64_t *>(smem + L.sbar);  // staging barriers: input, RMSNorm weight
  float *stg = reinterpret_cast<float *>(smem + L.stg);
  float *stw = reinterpret_cast<float *>(smem + L.stw);
  float *scr = reinterpret_cast<float *>(smem + L.scr);                                 // 64 floats
  unsigned long long *sbase = reinterpret_cast<unsigned long long *>(smem + L.scr + 256u);
  // unit-arrival counts of the KV heads at the step's start (kv_heads <= 64)
  unsigned long long *srdy = reinterpret_cast<unsigned long long *>(smem + L.scr + 512u);

  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
  uint32_t *err = p.ctrl + kCtrlErr;
  const uint32_t nb = p.pre + p.n_layers * kPhasesPerLayer;  // barriers per step = arrivals per CTA
  const uint32_t G = p.heads / p.kv_heads;

  if (threadIdx.x == 0) {
    for (uint32_t i = 0; i < R.nst; ++i) {
      mbar_init(&R.full[i], 1);
      mbar_init(&R.empty[i], kMvConsumers);
    }
    mbar_init(&sbar[0], 1);
    mbar_init(&sbar[1], 1);
    fence_mbar_init();
    // Every CTA arrives exactly nb times per step, so at a step's start the
    // counter is base + (arrivals of this step so far) with base a multiple of
    // nb * gridDim.x and fewer than nb * gridDim.x arrivals counted.
    // A nonzero kCtrlBarExtra raises every barrier target of this step beyond
    // what the grid provides, so the first wait runs out (the failure test);
    // every CTA still arrives nb times, which keeps the counter aligned.
    const unsigned long long c = ld_acquire_u64(p.bar);
    const unsigned long long unit = (unsigned long long)nb * gridDim.x;
    *sbase = c - c % unit + p.ctrl[kCtrlBarExtra];
  }
  for (uint32_t i = threadIdx.x; i < p.n_layers * (uint32_t)sizeof(StepLayer) / 8u; i += blockDim.x)
    reinterpret_cast<unsigned long long *>(layers)[i] = reinterpret_cast<const unsigned long long *>(p.layers)[i];
  // Read before this CTA's first grid-barrier arrival: the first release of
  // this step comes after the first barrier, which waits for every CTA.
  for (uint32_t i = threadIdx.x; i < p.kv_heads; i += blockDim.x) srdy[i] = ld_acquire_u64(p.ready + i);
  __syncthreads();
  const unsigned long long base = *sbase;

  uint32_t pos = p.ctrl[kCtrlPos];
  if (pos >= p.ctx) {
    if (threadIdx.x == 0) set_error(err, kErrPosition);
    pos = p.ctx - 1;
  }
  const uint32_t nch = (pos + 1u + p.chunk - 1u) / p.chunk;  // attention chunks per KV head
  const uint32_t n_units = p.kv_heads * nch;

  // ---------------- producer ----------------
  if (warp == kMvConsumers) {
    if (lane == 0) {
      RingPos rp;
      bool live = true;
      auto stream = [&](const uint8_t *w, const TileGeom &g) {
        if (!live) return;
        uint32_t t0, t1;
        tile_run(g, t0, t1);
        const uint32_t NSEG = g.nseg(), SEGB = g.seg_bytes();
        live = mv_produce(R, w + (uint64_t)t0 * NSEG * SEGB, (t1 - t0) * NSEG, SEGB, rp, err, err);
      };
      auto rows = [&](const __half *src, uint32_t n) {  // one stage of n cached K or V rows
        if (!live) return;
        live = ring_claim(R, rp, n * D * 2u, err, err);
        if (!live) return;
        if (n) bulk_g2s(R.ring + rp.slot * R.slot, src, n * D * 2u, &R.full[rp.slot]);
        rp.next(R.nst);
      };
      // the phases in order, each through one call site
      for (uint32_t ph = 0; ph <= nb && live; ++ph) {
        if (ph < p.pre) {
          if (ph == 2u) stream(p.w_fuse, p.g_fuse);
          else if (p.fsq_on) stream(ph == 0u ? p.w_fin : p.w_fout, ph == 0u ? p.g_fin : p.g_fout);
          continue;
        }
        const uint32_t l = (ph - p.pre) / kPhasesPerLayer, kind = ph - p.pre - l * kPhasesPerLayer;
        const StepLayer &Ly = layers[l < p.n_layers ? l : 0u];
        if (ph < nb && kind == kPhAttn) {
          for (uint32_t u = blockIdx.x; u < n_units; u += gridDim.x) {
            const AttnUnit a = attn_unit(p, u, nch, pos);
            for (uint32_t h = 0; h < 2; ++h) rows((h ? Ly.vc : Ly.kc) + ((size_t)a.kvh * p.ctx + a.r0) * D, a.staged);
          }
          continue;
        }
        if (ph == nb && !p.want_logits) break;
        const uint8_t *w = p.head;
        TileGeom g = p.g_head;
        if (ph < nb) {
          w = kind == kPhQkv ? Ly.qkv : kind == kPhO ? Ly.o : kind == kPhGu ? Ly.gateup : Ly.down;
          g = kind == kPhQkv ? p.g_qkv : kind == kPhO ? p.g_o : kind == kPhGu ? p.g_gu : p.g_down;
        }
        stream(w, g);
      }
      if (live) mv_drain(R, rp, err);
    }
    return;
  }

  // ---------------- consumers ----------------
  const uint32_t cw = warp, tid = cw * 32u + lane;
  RingPos rp;  // next ring stage
  bool ok = true;
  // Grid barrier before phase ph: every CTA has finished phase ph - 1.
  // ld.acquire.gpu in grid_wait, then the CTA barrier, orders every consumer
  // thread's later loads after the other CTAs' writes; red.release.gpu in
  // grid_arrive, after the CTA barrier, publishes every consumer thread's
  // writes of the phase (release is cumulative over what the barrier ordered).
  auto wait_phase = [&](uint32_t ph) {
    if (cw == 0 && lane == 0 && ph > 0 &&
        !grid_wait(p.bar, base + (unsigned long long)ph * gridDim.x, err))
      set_error(err, kErrGridWait);
    named_bar(1, NCT);
  };
  auto arrive = [&] {
    named_bar(1, NCT);
    if (cw == 0 && lane == 0) grid_arrive(p.bar);
  };
  uint32_t spar = 0;  // parities of the two staging barriers (bit 0 input, bit 1 RMSNorm weight)
  auto zero_red = [&](uint32_t tiles) {
    for (uint32_t i = cw * 32u + lane; i < tiles * kMvConsumers * kTileRows; i += NCT) red[i] = 0.f;
  };
  // One matvec phase over this CTA's tile run of g. Every matvec phase of the
  // step (and the final RMSNorm) goes through this one call site per weight
  // type, so the consumer code is a single copy that stays in the instruction
  // cache from phase to phase; the epilogue, the prologue and the input source
  // are runtime values.
  auto matvec = [&](auto q8c, Mode mode, bool rms, uint32_t ph, const MvParams &mp, const XSrc &src, float *xout,
                    bool consume) {
    constexpr bool WQ8 = decltype(q8c)::value;
    const TileGeom &g = mp.g;
    uint32_t t0, t1;
    tile_run(g, t0, t1);
    const uint32_t NSEG = g.nseg(), SEGB = g.seg_bytes();
    if (consume) zero_red(t1 - t0);
    const uint32_t C = g.cols;
    // the RMSNorm weight does not depend on the step: its copy starts before the wait
    if (rms && tid == 0) {
      mbar_arrive_expect_tx(sbar + 1, C * 4u);
      bulk_g2s(stw, mp.normw, C * 4u, sbar + 1);
    }
    // One bulk copy of the input, issued by the thread that acquired the other
    // CTAs' writes at the grid barrier as soon as it has them (it orders them
    // before its async-proxy read). stg is free: the CTA barrier that ended the
    // previous phase came after its last reader.
    if (tid == 0) {
      if (ph > 0 && !grid_wait(p.bar, base + (unsigned long long)ph * gridDim.x, err)) set_error(err, kErrGridWait);
      if (src.x != nullptr) {
        fence_proxy_async_global();
        mbar_arrive_expect_tx(sbar, C * 4u);
        bulk_g2s(stg, src.x, C * 4u, sbar);
      }
    }
    named_bar(1, NCT);
    if (src.x == nullptr) {
      for (uint32_t k = tid; k < C; k += NCT) stg[k] = xsrc_elem<true>(src, k);  // token-table row
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
    step_activation<WQ8>(C, NSEG * g.seg_cols(), rms, stg, stw, mp.eps, aux, p.plane, scr, cw, lane, xout);
    if (consume)
      mv_consume<WQ8>(R, rp, (t1 - t0) * NSEG, NSEG, SEGB, aux, p.plane, red, mp, t0, cw, lane, err, err, ok,
                      (rms && xout == nullptr) ? scr + 8 : nullptr,
                      [&](uint32_t R0) {  // the residual, in flight during the K loop
                        float2 v = make_float2(0.f, 0.f);
                        if (mode == Mode::RESID || mode == Mode::FSQ) {
                          if (R0 < mp.g.rows) v.x = __ldcg(mp.resid + R0);
                          if (R0 + 8u < mp.g.rows) v.y = __ldcg(mp.resid + R0 + 8u);
                        }
                        return v;
                      },
                      [&](uint32_t R0, float a, float b, float2 pv) {
                        switch (mode) {
                          case Mode::PLAIN: mv_epilogue<Mode::PLAIN>(mp, R0, a, b, pos); break;
                          case Mode::RESID: {  // residual_rmsnorm.comp:27 (linear_bias.comp:75 with alpha 1)
                            const float y0 = __fadd_rn(pv.x, __fmul_rn(a, mp.alpha));
                            const float y1 = __fadd_rn(pv.y, __fmul_rn(b, mp.alpha));
                            if (R0 < mp.g.rows) mp.out[R0] = y0;
                            if (R0 + 8u < mp.g.rows) mp.out[R0 + 8u] = y1;
                            if (mp.out2) {
                              if (R0 < mp.g.rows) mp.out2[R0] = y0;
                              if (R0 + 8u < mp.g.rows) mp.out2[R0 + 8u] = y1;
                            }
                            break;
                          }
                          case Mode::FSQ: {  // linear_bias.comp:75, then fsq_quantize.comp:8-11
                            const float s = p.fsq_scale;
                            if (R0 < mp.g.rows)
                              mp.out[R0] = __fdiv_rn(roundf(__fmul_rn(tanhf(__fadd_rn(pv.x, a)), s)), s);
                            if (R0 + 8u < mp.g.rows)
                              mp.out[R0 + 8u] = __fdiv_rn(roundf(__fmul_rn(tanhf(__fadd_rn(pv.y, b)), s)), s);
                            break;
                          }
                          case Mode::SWIGLU: mv_epilogue<Mode::SWIGLU>(mp, R0, a, b, pos); break;
                          case Mode::QKV: mv_epilogue<Mode::QKV>(mp, R0, a, b, pos); break;
                        }
                      });
  };

  uint32_t tok = 0;
  if (p.token_input) {
    tok = p.ctrl[kCtrlToken];
    if (tok >= p.g_tok.rows) {
      if (cw == 0 && lane == 0) set_error(err, kErrBadToken);
      tok = 0;
    }
  }

  // Phases nb * layer + kind, then phase nb: the final RMSNorm and the optional LM head.
  for (uint32_t ph = 0; ph <= nb; ++ph) {
    const uint32_t lp = ph < p.pre ? 0u : ph - p.pre;  // phase within the layers
    const uint32_t l = lp / kPhasesPerLayer;
    const uint32_t kind = lp - l * kPhasesPerLayer;
    const StepLayer &Ly = layers[l < p.n_layers ? l : 0u];

    // ---- attention: split-K units, then one merge slice per query head ----
    if (ph >= p.pre && ph < nb && kind == kPhAttn) {
      wait_phase(ph);
      constexpr uint32_t KS = D / 16u;              // K-steps of a head row
      const uint32_t HT = (G + 7u) / 8u;            // tiles of 8 heads
      const uint32_t SST = p.chunk + 4u;            // row stride of sS (padded)
      uint2 *sQB = reinterpret_cast<uint2 *>(aux);  // [HT][KS][2][32] q fragments
      float *sS = reinterpret_cast<float *>(aux + HT * KS * 2u * 32u * 8u);  // [G][SST]
      static_assert(D / 2u <= NCT, "one word of the current K and V row per thread");
      for (uint32_t u = blockIdx.x; u < n_units; u += gridDim.x) {
        const AttnUnit a = attn_unit(p, u, nch, pos);
        // the current position's K and V rows (stored by this step's QKV phase)
        // are loaded here, so their L2 round trip overlaps the q loads below
        const bool cur_row = a.staged < a.len && tid < D / 2u;
        uint32_t kcur = 0, vcur = 0;
        if (cur_row) {
          kcur = __ldcg(reinterpret_cast<const unsigned int *>(Ly.kc + ((size_t)a.kvh * p.ctx + pos) * D) + tid);
          vcur = __ldcg(reinterpret_cast<const unsigned int *>(Ly.vc + ((size_t)a.kvh * p.ctx + pos) * D) + tid);
        }
        // q of the group as the B operand of the score MMAs (K = dims, N = 8
        // heads per tile), split into fp16 hi + lo: entry [ht][ks][h][lane] =
        // the lane's b0/b1 words (rows 2tq, 2tq+1 and 2tq+8, 2tq+9 of K-step
        // ks, column gq = head ht * 8 + gq); heads beyond G are zero
        for (uint32_t e = tid; e < HT * KS * 32u; e += NCT) {
          const uint32_t ln = e & 31u, ks = (e >> 5) % KS, ht = (e >> 5) / KS;
          const uint32_t g = ht * 8u + (ln >> 2), d0 = ks * 16u + (ln & 3u) * 2u;
          float v[4] = {0.f, 0.f, 0.f, 0.f};
          if (g < G) {
            const float *qg = p.q + ((size_t)a.kvh * G + g) * D + d0;
            v[0] = __ldcg(qg);
            v[1] = __ldcg(qg + 1);
            v[2] = __ldcg(qg + 8);
            v[3] = __ldcg(qg + 9);
          }
          uint32_t hw[2], lw[2];
#pragma unroll
          for (int j = 0; j < 2; ++j) {
            const __half h0 = __float2half_rn(v[2 * j]), h1 = __float2half_rn(v[2 * j + 1]);
            const __half l0 = __float2half_rn(v[2 * j] - __half2float(h0));
            const __half l1 = __float2half_rn(v[2 * j + 1] - __half2float(h1));
            hw[j] = pack_half2(h0, h1);
            lw[j] = pack_half2(l0, l1);
          }
          sQB[((ht * KS + ks) * 2u + 0u) * 32u + ln] = make_uint2(hw[0], hw[1]);
          sQB[((ht * KS + ks) * 2u + 1u) * 32u + ln] = make_uint2(lw[0], lw[1]);
        }
        const uint32_t sK = rp.slot, pK = rp.phase;
        rp.next(R.nst);
        const uint32_t sV = rp.slot, pV = rp.phase;
        rp.next(R.nst);
        if (!mbar_wait_bounded(&R.full[sK], pK, err) || !mbar_wait_bounded(&R.full[sV], pV, err)) {
          set_error(err, kErrConsumerWait);
          ok = false;
        }
        __half *kS = reinterpret_cast<__half *>(R.ring + sK * R.slot);
        __half *vS = reinterpret_cast<__half *>(R.ring + sV * R.slot);
        const uint32_t len16 = (a.len + 15u) & ~15u;
        if (cur_row) {
          reinterpret_cast<uint32_t *>(kS + a.staged * D)[tid] = kcur;
          reinterpret_cast<uint32_t *>(vS + a.staged * D)[tid] = vcur;
        }
        // V rows past the chunk's end meet zero weights; make them zero too (not
        // stale bytes, which may be NaN)
        for (uint32_t i = a.len * D / 2u + tid; i < len16 * D / 2u; i += NCT) reinterpret_cast<uint32_t *>(vS)[i] = 0u;
        named_bar(1, NCT);
        // scores (attn_scores.comp:27-44): S[t][g] = K[t] . q[g] on the tensor
        // cores, a warp per (16 positions, 8 heads) tile
        for (uint32_t it = cw; it < (len16 / 16u) * HT; it += kMvConsumers) {
          const uint32_t pt = it / HT, ht = it % HT;
          float c[4] = {0.f, 0.f, 0.f, 0.f}, cl[4] = {0.f, 0.f, 0.f, 0.f};  // hi and lo chains
          const uint32_t kt = pt * 16u + (lane & 15u);  // this lane's K row (chunk-permuted, kv_swz)
          const __half *kb = kS + kt * D;
#pragma unroll 4
          for (uint32_t ks = 0; ks < KS; ++ks) {
            uint32_t af[4];
            ldmatrix_x4(af, kb + kv_swz(a.r0 + kt, (lane >> 4) * 8u + ks * 16u, D));
            const uint2 bh = sQB[((ht * KS + ks) * 2u + 0u) * 32u + lane];
            const uint2 bl = sQB[((ht * KS + ks) * 2u + 1u) * 32u + lane];
            mma_f16(c, af, bh.x, bh.y);
            mma_f16(cl, af, bl.x, bl.y);
          }
          const uint32_t t = pt * 16u + (lane >> 2), g = ht * 8u + (lane & 3u) * 2u;
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const uint32_t tt = t + (j >> 1) * 8u, gg = g + (j & 1);
            if (tt < a.len && gg < G) sS[gg * SST + tt] = __fmul_rn(__fadd_rn(c[j], cl[j]), p.attn_scale);
          }
        }
        named_bar(1, NCT);
        // chunk softmax (softmax.comp): warp per head; exp(s - m) replaces s
        for (uint32_t g0 = cw; g0 < G; g0 += kMvConsumers) {
          float *sg = sS + g0 * SST;
          float m = -INFINITY;
          for (uint32_t t = lane; t < a.len; t += 32) m = fmaxf(m, sg[t]);
          m = warp_max(m);
          float lsum = 0.f;
          for (uint32_t t = lane; t < a.len; t += 32) {
            const float e = expf(sg[t] - m);
            sg[t] = e;
            lsum += e;
          }
          lsum = warp_sum(lsum);
          if (lane == 0) {
            const size_t slot_i = ((size_t)a.kvh * p.max_chunks + a.c) * G + g0;
            p.part_ml[slot_i] = make_float2(m, lsum);
          }
        }
        named_bar(1, NCT);
        // values (attn_values.comp): O[g][d] = sum_t P[g][t] V[t][d] as
        // (V^T)(P^T) on the tensor cores, a warp per (16 dims, 8 heads) tile;
        // A = V^T from the V rows by transposing loads, B = P^T in fp16 hi + lo
        for (uint32_t it = cw; it < KS * HT; it += kMvConsumers) {
          const uint32_t dt = it / HT, ht = it % HT;
          float c[4] = {0.f, 0.f, 0.f, 0.f}, cl[4] = {0.f, 0.f, 0.f, 0.f};  // hi and lo chains
          const uint32_t gb = ht * 8u + (lane >> 2);  // head of this lane's B column
          const float *pg = sS + (gb < G ? gb : 0u) * SST;
          const uint32_t vt = ((lane >> 4) & 1u) * 8u + (lane & 7u);  // this lane's V row in each 16 (kv_swz)
          const uint32_t ve = dt * 16u + ((lane >> 3) & 1u) * 8u;
          for (uint32_t kk = 0; kk < len16 / 16u; ++kk) {
            uint32_t af[4];
            ldmatrix_x4_trans(af, vS + (kk * 16u + vt) * D + kv_swz(a.r0 + kk * 16u + vt, ve, D));
            float w[4];
            const uint32_t t0w = kk * 16u + (lane & 3u) * 2u;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const uint32_t tt = t0w + (j & 1) + (j >> 1) * 8u;
              w[j] = (gb < G && tt < a.len) ? pg[tt] : 0.f;
            }
            uint32_t bh[2], bl[2];
#pragma unroll
            for (int j = 0; j < 2; ++j) {
              const __half h0 = __float2half_rn(w[2 * j]), h1 = __float2half_rn(w[2 * j + 1]);
              bh[j] = pack_half2(h0, h1);
              bl[j] = pack_half2(__float2half_rn(w[2 * j] - __half2float(h0)),
                                 __float2half_rn(w[2 * j + 1] - __half2float(h1)));
            }
            mma_f16(c, af, bh[0], bh[1]);
            mma_f16(cl, af, bl[0], bl[1]);
          }
          // c: dims dt * 16 + gq (+ 8), heads ht * 8 + 2tq (+ 1)
          const uint32_t d = dt * 16u + (lane >> 2), g = ht * 8u + (lane & 3u) * 2u;
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const uint32_t dd = d + (j >> 1) * 8u, gg = g + (j & 1);
            if (gg < G) p.part[(((size_t)a.kvh * p.max_chunks + a.c) * G + gg) * D + dd] = __fadd_rn(c[j], cl[j]);
          }
        }
        // every warp is done with the K and V stages, and every partial of the
        // unit is written (the barrier orders those writes before the unit's
        // release)
        named_bar(1, NCT);
        if (lane == 0) {
          mbar_arrive(&R.empty[sK]);
          mbar_arrive(&R.empty[sV]);
        }
        // this unit's partials are written: one arrival at its KV head
        if (cw == 0 && lane == 0) grid_arrive(p.ready + a.kvh);
        named_bar(1, NCT);  // sQB / sS reuse by the next unit
      }
      // Merge slices, one query head each, on the CTAs from the end of the
      // grid (free of units while n_units <= gridDim.x - heads): wait for all
      // nch arrivals of the head's units in this layer (the acquire that reads
      // the last one synchronises with every unit's release), then
      // o = sum_c exp(m_c - M) o_c / sum_c exp(m_c - M) l_c
      // over its chunks. Thread (grp, col) sums float4 column col of the chunks
      // grp, grp + NGR, ...; the groups' rows are then added in order.
      for (uint32_t j = gridDim.x - 1u - blockIdx.x; j < p.heads; j += gridDim.x) {
        const uint32_t kvh = j / G, g0 = j - kvh * G;
        if (cw == 0 && lane == 0 && !grid_wait(p.ready + kvh, srdy[kvh] + (unsigned long long)(l + 1u) * nch, err)) set_error(err, kErrGridWait);
        named_bar(1, NCT);
        constexpr uint32_t NCOL = D / 4u, NGR = NCT / NCOL, MR = 8u;  // columns, chunk groups, rows in flight
        static_assert(NCT % NCOL == 0, "whole chunk groups");
        float *sW = reinterpret_cast<float *>(aux);  // [max_chunks] weights, then 1/sum
        float4 *sO = reinterpret_cast<float4 *>(aux + step_merge_w_bytes(p.max_chunks));
        const uint32_t col = tid % NCOL, grp = tid / NCOL;
        const size_t hb = (size_t)kvh * p.max_chunks * G + g0;  // slot of chunk 0
        const float4 *ob = reinterpret_cast<const float4 *>(p.part + hb * D) + col;
        auto row = [&](uint32_t c) { return __ldcg(ob + (size_t)c * G * NCOL); };
        // the first MR rows of this thread's chunks load with the weights
        float4 v[MR];
#pragma unroll
        for (uint32_t i = 0; i < MR; ++i) {
          const uint32_t c = grp + i * NGR;
          v[i] = c < nch ? row(c) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
        if (cw == 0) {
          constexpr uint32_t MLR = 4u;  // (max, sum) pairs per lane held in registers
          float2 ml[MLR];
          float M = -INFINITY;
#pragma unroll
          for (uint32_t i = 0; i < MLR; ++i) {
            const uint32_t c = lane + 32u * i;
            ml[i] = c < nch ? __ldcg(&p.part_ml[hb + (size_t)c * G]) : make_float2(-INFINITY, 0.f);
            M = fmaxf(M, ml[i].x);
          }
          for (uint32_t c = lane + 32u * MLR; c < nch; c += 32u) M = fmaxf(M, __ldcg(&p.part_ml[hb + (size_t)c * G]).x);
          M = warp_max(M);
          float Ls = 0.f;
#pragma unroll
          for (uint32_t i = 0; i < MLR; ++i) {
            const uint32_t c = lane + 32u * i;
            if (c < nch) {
              const float w = ml[i].x == -INFINITY ? 0.f : expf(ml[i].x - M);
              sW[c] = w;
              Ls = fmaf(w, ml[i].y, Ls);
            }
          }
          for (uint32_t c = lane + 32u * MLR; c < nch; c += 32u) {
            const float2 m2 = __ldcg(&p.part_ml[hb + (size_t)c * G]);
            const float w = m2.x == -INFINITY ? 0.f : expf(m2.x - M);
            sW[c] = w;
            Ls = fmaf(w, m2.y, Ls);
          }
          Ls = warp_sum(Ls);
          if (lane == 0) sW[p.max_chunks] = 1.0f / Ls;
        }
        named_bar(1, NCT);
        float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
        auto acc = [&](uint32_t c, const float4 &r) {
          const float w = sW[c];
          o.x = fmaf(w, r.x, o.x);
          o.y = fmaf(w, r.y, o.y);
          o.z = fmaf(w, r.z, o.z);
          o.w = fmaf(w, r.w, o.w);
        };
#pragma unroll
        for (uint32_t i = 0; i < MR; ++i)
          if (grp + i * NGR < nch) acc(grp + i * NGR, v[i]);
        for (uint32_t c = grp + MR * NGR; c < nch; c += NGR) acc(c, row(c));
        sO[grp * NCOL + col] = o;
        named_bar(1, NCT);
        if (tid < NCOL) {
          float4 t = sO[tid];
          for (uint32_t gi = 1; gi < NGR; ++gi) {
            const float4 u = sO[gi * NCOL + tid];
            t.x += u.x;
            t.y += u.y;
            t.z += u.z;
            t.w += u.w;
          }
          const float inv = sW[p.max_chunks];
          reinterpret_cast<float4 *>(p.attn + ((size_t)kvh * G + g0) * D)[tid] =
              make_float4(t.x * inv, t.y * inv, t.z * inv, t.w * inv);
        }
        named_bar(1, NCT);  // sW / sO reuse
      }
      arrive();
      continue;
    }

    MvParams mp{};
    mp.ctrl = p.ctrl;
    mp.eps = p.eps;
    XSrc src{};
    Mode mode = Mode::PLAIN;
    bool rms = false, consume = true;
    float *xout = nullptr;
    if (ph < p.pre) {
      // ResidualLM: linear_bias.comp (+ fsq_quantize.comp) and fusion_linear.comp
      if (ph < 2u && !p.fsq_on) {
        wait_phase(ph);
        arrive();
        continue;
      }
      mp.alpha = 1.0f;
      if (ph == 0u) {
        mp.g = p.g_fin;
        mp.out = p.fsq_lat;
        mp.resid = p.b_fin;
        src.x = p.res_base;
        mode = Mode::FSQ;
      } else if (ph == 1u) {
        mp.g = p.g_fout;
        mp.out = p.fuse_in;
        mp.out2 = p.fsq_res;
        mp.resid = p.b_fout;
        src.x = p.fsq_lat;
        mode = Mode::RESID;
      } else {
        mp.g = p.g_fuse;
        mp.out = p.hid_a;
        mp.out2 = p.fused;
        mp.resid = p.b_fuse;
        src.x = p.fuse_in;
        mode = Mode::RESID;
      }
    } else if (ph == nb) {
      // final RMSNorm into out (CTA 0), and the LM head on it when logits are wanted
      if (!p.want_logits && blockIdx.x != 0) break;
      mp.g = p.want_logits ? p.g_head : p.g_qkv;
      mp.normw = p.out_norm;
      mp.out = p.logits;
      mp.alpha = p.logit_scale;
      src.x = p.hid_a;
      rms = true;
      consume = p.want_logits != 0;
      xout = blockIdx.x == 0 ? p.out : nullptr;
    } else if (kind == kPhQkv) {
      // QKV + RoPE + KV store on RMSNorm(hid_a), or of the token's embedding row
      mp.g = p.g_qkv;
      mp.normw = Ly.attn_norm;
      mp.out = p.q;
      mp.q_rows = p.H;
      mp.kv_rows = p.kv_heads * p.head_dim;
      mp.head_dim = p.head_dim;
      mp.ctx = p.ctx;
      mp.kc = Ly.kc;
      mp.vc = Ly.vc;
      mp.inv_freq = p.inv_freq;
      mp.ext = p.ext;
      mp.rope_scaling = p.rope_scaling;
      mode = Mode::QKV;
      rms = true;
      if (l == 0 && p.token_input) {
        src.tab = p.tok;
        src.g = p.g_tok;
        src.token = tok;
        src.alpha = p.emb_scale;
        // every CTA dequantises the row itself; CTA 0 also stores it as the residual stream
        if (blockIdx.x == 0)
          for (uint32_t k = cw * 32u + lane; k < p.H; k += NCT) p.hid_a[k] = xsrc_elem<true>(src, k);
      } else {
        src.x = p.hid_a;
      }
    } else if (kind == kPhO) {
      // o_proj + residual: hid_b = hid_a + scale * O attn
      mp.g = p.g_o;
      mp.out = p.hid_b;
      mp.resid = p.hid_a;
      mp.alpha = p.res_scale;
      src.x = p.attn;
      mode = Mode::RESID;
    } else if (kind == kPhGu) {
      // gate/up + SwiGLU on RMSNorm(hid_b)
      mp.g = p.g_gu;
      mp.normw = Ly.ffn_norm;
      mp.out = p.gate;
      src.x = p.hid_b;
      mode = Mode::SWIGLU;
      rms = true;
    } else {
      // down + residual: hid_a = hid_b + scale * Down gate
      mp.g = p.g_down;
      mp.out = p.hid_a;
      mp.resid = p.hid_b;
      mp.alpha = p.res_scale;
      src.x = p.gate;
      mode = Mode::RESID;
    }
    if (mp.g.q8 != Q8) {
      // an LM head in the other weight format runs as its own launch after this one
      if (cw == 0 && lane == 0) set_error(err, kErrPlan);
      mp.g = p.g_qkv;
      consume = false;
    }
    matvec(std::integral_constant<bool, Q8>{}, mode, rms, ph, mp, src, xout, consume);
    if (ph < nb) arrive();
  }
  if (blockIdx.x == 0) {
    named_bar(1, NCT);
    if (cw == 0 && lane == 0) p.ctrl[kCtrlPos] = pos + 1u;
  }
}

}  // namespace vg
