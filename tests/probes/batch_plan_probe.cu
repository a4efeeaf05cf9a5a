// Host-side check of the batched kernel's attention plan (test infrastructure,
// built and run by tests/test_cpu_batch_plan.py; no GPU). For every model shape
// the batched kernel takes (head_dim 32 / 64 / 128, an even group of up to 8
// query heads, up to 8 KV heads), every column count 1..16 and several SM
// counts, it checks the merge-slice width that batch_merge_width picks against
// what the merge loop in decode_batch_kernel relies on:
//  - the width divides head_dim and is at least 16;
//  - a slice's threads (width x group / heads loaded at once) fit the 256
//    consumer threads, and every (dimension, head group) of the slice has a
//    thread with a chunk part;
//  - the parts' outputs fit the area batch_attn_bytes reserves after the
//    chunk weights and the partial maxima / sums;
//  - the loads stay aligned to the heads loaded at once (16 or 8 bytes);
//  - more slices than CTAs only when no wider slice is allowed, and the
//    narrowest width that fits otherwise.
// Prints "ok <cases>" or the first violation.
#include <cstdio>
#include <cstdint>
#include <cstdlib>

#include "../../voxgen_b200/csrc/batch_kernel.cuh"

int main() {
  using namespace vg;
  const uint32_t NCT = kMvConsumers * 32u;
  unsigned long cases = 0;
  for (uint32_t D : {32u, 64u, 128u})
    for (uint32_t G = 2; G <= 8; G += 2)
      for (uint32_t kvh = 1; kvh <= 8; ++kvh)
        for (uint32_t S = 1; S <= kBatchMaxCols; ++S)
          for (uint32_t grid : {100u, 132u, 148u, 160u}) {
            ++cases;
            const uint32_t dw = batch_merge_width(S, kvh, D, G, grid);
            // the merge loop's mapping (decode_batch_kernel, merge slices)
            const uint32_t VW = G % 4u == 0 ? 4u : 2u, GV = G / VW, TPR = dw * GV;
            if (dw < 16u || D % dw) {
              printf("bad width %u for head_dim %u\n", dw, D);
              return 1;
            }
            if (G % VW || TPR > NCT) {
              printf("slice threads %u > %u (G %u, width %u)\n", TPR, NCT, G, dw);
              return 1;
            }
            const uint32_t NPART = NCT / TPR;
            // every (dl, hq) pair is owned by the threads of part 0
            for (uint32_t rr = 0; rr < TPR; ++rr) {
              const uint32_t dl = rr / GV, hq = rr % GV;
              if (dl >= dw || hq * VW + VW > G) {
                printf("thread %u maps outside the slice (G %u width %u)\n", rr, G, dw);
                return 1;
              }
              // float offset of the load inside a chunk's [D][G] block
              const uint32_t off = dl * G + hq * VW;
              if (off % VW) {
                printf("misaligned load at float %u (G %u)\n", off, G);
                return 1;
              }
            }
            // parts' outputs after sW [max_chunks][8], sM [32][8], sS [32][8]
            const uint32_t max_chunks = 1024u;
            const uint32_t need = (max_chunks * 8u + 512u + NPART * dw * G) * 4u;
            if (need > batch_attn_bytes(batch_chunk(D), max_chunks)) {
              printf("merge scratch %u > %u bytes (G %u width %u)\n", need, batch_attn_bytes(batch_chunk(D), max_chunks),
                     G, dw);
              return 1;
            }
            // more slices than CTAs only when no wider slice is allowed, and no
            // wider slice than needed
            const bool can_widen = dw < D && 2u * dw * GV <= NCT;
            if (can_widen && S * kvh * (D / dw) > grid) {
              printf("width %u leaves %u slices for %u CTAs\n", dw, S * kvh * (D / dw), grid);
              return 1;
            }
            if (dw > 16u && S * kvh * (D / (dw / 2u)) <= grid) {
              printf("width %u where %u would fit %u CTAs\n", dw, dw / 2u, grid);
              return 1;
            }
          }
  printf("ok %lu\n", cases);
  return 0;
}
