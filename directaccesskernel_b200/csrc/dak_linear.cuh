// dak_linear.cuh - launch parameters shared by the split-tier linear kernels.
//
// Data layout (kept from the reference, app/python/layers/linearLayer.py:226-229):
// each tier holds the transposed weight Wt[K, cols] row-major, output features
// contiguous, so one weight row segment of 64 features is 128 contiguous bytes.
// The host tier lives in pinned, mapped host memory and is read by the GPU over
// the host link; the device tier lives in HBM.  Both are streamed through the
// same shared-memory ring by TMA tile loads, never staged through HBM.
#pragma once

#include <cuda.h>
#include <stdint.h>

namespace dak {

constexpr int kBoxCols = 64;  // 64 x 16-bit = 128 B = one 128-byte swizzle span

// ---- CUDA-core decode kernel (ntok <= 8) ---------------------------------
// Stage shapes follow a measured rule of this part: TMA streams a [K, N]
// weight at 6.0-6.5 TB/s with boxes of 8-16 KB (64 x 64 or 64 x 128), but at
// 3.5 TB/s with 4 KB boxes.  Both kernels use 128-feature x 128-row stages (two
// 16 KB boxes), so narrow layers still have enough whole tiles to spread.
constexpr int kCoreBN = 128;                      // output features per tile (2 boxes)
constexpr int kCoreBoxes = kCoreBN / kBoxCols;    // TMA boxes per stage
constexpr int kCoreBK = 128;                      // K rows per stage (16 KB boxes)
constexpr int kCoreStages = 6;                    // most weight stages (32 KB each)
static_assert(kCoreBoxes == 2 && kCoreBK == 128, "the consumer warp map covers 2 boxes x 2 row halves of 64");
constexpr int kCoreConsumerWarps = 8;
constexpr int kCoreThreads = (kCoreConsumerWarps + 1) * 32;
constexpr int kCoreMaxTok = 8;
// Automatic path choice: the CUDA-core kernel up to this many tokens, tcgen05
// above.  Measured on B200 over the Llama-3-8B shapes (back-to-back launches,
// HBM only): CUDA core 78.9 / 84.8 / 105.7 / 146.2 us at 1 / 2 / 4 / 8 tokens,
// tcgen05 86.9 us at 16 tokens.  From 3 tokens up, the FP32 FMA work of
// the CUDA-core kernel, not the weight stream, sets its time.
constexpr int kCoreAutoMaxTok = 2;

// ---- tcgen05 kernel (ntok up to 256) --------------------------------------
constexpr int kMmaBM = 128;                       // UMMA M: output features per tile (2 boxes)
constexpr int kMmaBK = 128;                       // K rows per stage (8 x UMMA K=16; 16 KB boxes)
constexpr int kMmaMaxTok = 256;                   // UMMA N limit
constexpr int kMmaEpiWarps = 4;
constexpr int kMmaThreads = (2 + kMmaEpiWarps) * 32;  // producer, MMA, 4 epilogue

struct alignas(64) LinearTier {
  CUtensorMap wmap;  // Wt[K, cols]; box {64, BK}; 128-byte swizzle
  int cols;          // output features of this tier
  int col_offset;    // first output column of this tier in y
  int cta_begin;     // CTAs [cta_begin, cta_begin + cta_count) serve this tier
  int cta_count;
  int ksplit;        // CTAs (consecutive, same cluster) sharing one tile along K
  int pad_[3];
};

// Work of group g (ksplit consecutive CTAs) of a tier with `groups` groups:
// the contiguous 64-feature boxes [box_begin, box_end), split evenly so that
// no group gets more than one box above the average, walked as tiles of up to
// `boxes_per_tile` boxes; every CTA of the group covers its own K range.
struct GroupWork {
  int box_begin, box_end, ntiles;
  __host__ __device__ GroupWork(int cols, int groups, int g, int boxes_per_tile) {
    const int boxes = (cols + kBoxCols - 1) / kBoxCols;
    box_begin = (int)((long long)g * boxes / groups);
    box_end = (int)((long long)(g + 1) * boxes / groups);
    ntiles = (box_end - box_begin + boxes_per_tile - 1) / boxes_per_tile;
  }
};

// Row-parallel all-reduce fused into the tcgen05 linear kernel (one-shot, over
// peer memory).  Every rank holds, in memory mapped into all ranks, a receive
// buffer of 2 parities x world slots of [ntok, ldy] 16-bit partials and a flag
// array of [max_ctas][world] epochs.  Call e (e = *epoch + 1) writes its
// partial outputs into slot `rank` of parity e & 1 on every rank, sets flag
// [cta][rank] = e on every rank (system-scope release), waits until every
// rank's flag [cta][*] reached e (bounded), and sums the slots into y.  The
// last CTA to finish bumps *epoch.  All ranks run the same shapes, hence the
// same plan, and the grid is one resident wave, so peer CTAs run together.
constexpr int kArMaxRanks = 8;
constexpr int kArMaxCtas = 1024;
// With a multicast mapping (NVSwitch), the partials instead stay local: call e
// stores its FP32 partials in this rank's own buffer (parity e & 1), publishes
// the flags, and reads the sum over ranks with multimem.ld_reduce through the
// multicast address, so each rank moves its data across NVLink once.
struct ArParams {
  uint16_t *buf[kArMaxRanks];    // each rank's receive buffer (this process's mapping)
  uint32_t *flags[kArMaxRanks];  // each rank's flag array
  float *own;                    // multicast mode: this rank's 2 x slot_elems FP32 buffer
  float *mc;                     // multicast mode: the same buffer's multicast address
  long long slot_elems;          // 16-bit elements per slot
  int *epoch;                    // this rank's call counter (device memory)
  int *done;                     // this rank's finished-CTA counter
  int world, rank;
  long long timeout_ns;
  int publish_only;              // multicast mode: store and publish; the consumer reduces
  int pad_;
};

struct alignas(64) LinearParams {
  LinearTier tier[2];  // [0] host tier, [1] device tier
  CUtensorMap xmap;    // x[ntok, K] activations
  void *y;             // y[ntok, ldy]
  long long ldy;
  int ntok;
  int K;
  int *status;         // device error word
  int red_slots;       // partial-sum slots reserved in shared memory (max ksplit - 1)
  int stages;          // pipeline depth (tcgen05 kernel; sized to the shared memory left)
  int pdl;             // launched with programmatic stream serialization: weights are
                       // prefetched before griddepcontrol.wait, x and y only after it
  int ar_on;           // 1: y is the all-reduce (sum over ranks) of this kernel's result
  int tok_slices;      // tcgen05 kernel: grid rows; row j serves tokens [j * NTOKP, (j+1) * NTOKP)
                       // of every tile (0 or 1: one row, all tokens)
  int glu;             // tcgen05 kernel: y = silu(gate) * up of gate/up rows interleaved in
                       // 16-feature blocks (y has half the weight's output features)
  ArParams ar;
};

}  // namespace dak
