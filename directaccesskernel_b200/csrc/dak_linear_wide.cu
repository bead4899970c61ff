// dak_linear_wide.cu - split-tier offloaded linear for 257..512 tokens on the
// tcgen05 tensor cores, streaming every weight tile once for the whole batch.
//
// Replaces, for batches above 256 tokens with host-resident weight rows, the
// reference's prefill kernels `gemv_multicast_prefill` and
// `gemv_horizontal_multicast_prefill` (include/task/gemv_multicast.cuh:601-914,
// selected by app/python/layers/linearLayerMulticast.py:121-124), which walk
// 256-token activation tiles.  The 256-token kernel (dak_linear_mma.cu) would
// take such a batch in two launches and read the weight twice; over the host
// link that doubles the time.  Here one CTA owns 128-feature tiles: per 64-row
// K stage it loads the two 64-feature weight boxes (8 KB each) and both token
// halves of the activations (two 256 x 64 boxes, 32 KB each), and one thread
// issues 4 K-steps x 2 halves of UMMA 128 x 256 x 16 into two 256-column FP32
// accumulators that together fill the SM's 512 TMEM columns.  Token t of the
// batch is accumulator column t.
//
// Paired mode (PAIR = true), for HBM-only layers wide enough to fill the SMs:
// the roles of the two operands swap.  A CTA owns two 128-feature tiles (four
// 64-feature boxes) and one 256-token row of the batch (grid row
// blockIdx.y), and applies each activation stage to both weight tiles: per
// 64-row K stage it loads four 8 KB weight boxes and one 32 KB activation box,
// and issues UMMA 128 x 256 x 16 once per tile into two 256-column
// accumulators.  Per K row of two tiles it moves 512 bytes of weights and 512
// of activations, where two separate tiles of the 256-token kernel move 512
// and 1024.  Three stages (64 KB each) fit.
//
// Roles (192 threads) as in the 256-token kernel: warp 0 issues TMA loads,
// warp 1 owns TMEM and issues the MMAs, warps 2..5 read the accumulators back
// (each its TMEM lane quadrant) and store the 16-bit output.  No split-K and
// no clusters: the CTAs of each tier walk an even share of whole 64-feature
// boxes.  With one accumulator set per CTA, the next tile's MMAs wait for the
// epilogue of the previous one; the weight stream, which bounds the host tier,
// keeps running meanwhile.
#include "dak_common.cuh"
#include "dak_host.h"
#include "dak_linear.cuh"
#include "dak_tcgen05.cuh"

namespace dak {

namespace {

constexpr int kWideBK = 64;                                   // K rows per stage (4 UMMA K-steps)
constexpr int kWideHalf = 256;                                // tokens per accumulator (UMMA N)
constexpr uint32_t kWideWBox = kBoxCols * kWideBK * 2;        // 8 KB: 64 features x 64 K rows
constexpr uint32_t kWideXBox = kWideHalf * kWideBK * 2;       // 32 KB: 256 tokens x 64 K
constexpr uint32_t kWideTmemCols = 2 * kWideHalf;             // 512: the whole TMEM

// Per mode: weight boxes and activation boxes per stage, and the stage count.
template <bool PAIR>
struct WideLayout {
  static constexpr int stages = PAIR ? 3 : 2;
  static constexpr int w_boxes = PAIR ? 4 : 2;                // 64-feature boxes per tile (the CTA's unit)
  static constexpr int x_boxes = PAIR ? 1 : 2;                // 256-token activation boxes per stage
  static constexpr uint32_t w_stage = w_boxes * kWideWBox;    // 32 KB / 16 KB
  static constexpr uint32_t x_stage = x_boxes * kWideXBox;    // 32 KB / 64 KB
  static constexpr uint32_t w_off = 0;
  static constexpr uint32_t x_off = w_off + stages * w_stage;
  static constexpr uint32_t bar_off = x_off + stages * x_stage;
  // full[S], empty[S], tmem_full, tmem_empty, last_done
  static constexpr uint32_t misc_off = bar_off + (2 * stages + 3) * 8;  // tmem slot, abort flags
  static constexpr uint32_t bytes = misc_off + 16 + 1024;                // + alignment slack
};
static_assert(WideLayout<false>::bytes <= 227 * 1024 && WideLayout<true>::bytes <= 227 * 1024,
              "the wide stages must fit one CTA's shared memory");
static_assert(WideLayout<false>::x_off % 1024 == 0 && WideLayout<true>::x_off % 1024 == 0 &&
                  kWideXBox % 1024 == 0 && kWideWBox % 1024 == 0,
              "128-byte-swizzled operand tiles start on 1024-byte boundaries");

template <typename T, bool PAIR>
__global__ void __launch_bounds__(kMmaThreads, 1) linear_wide_kernel(const __grid_constant__ LinearParams p) {
  using L = WideLayout<PAIR>;
  constexpr int S = L::stages;
  constexpr int kWideBoxesPerTile = L::w_boxes;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_u32 = smem_u32(smem_raw);
  uint8_t *smem = smem_raw + (((raw_u32 + 1023u) & ~1023u) - raw_u32);
  const uint32_t sbase = smem_u32(smem);

  const int warp = warp_id();
  const int lane = lane_id();

  const int ti = (p.tier[1].cta_count > 0 && (int)blockIdx.x >= p.tier[1].cta_begin) ? 1 : 0;
  const LinearTier &tier = p.tier[ti];
  const int local = (int)blockIdx.x - tier.cta_begin;
  const bool idle = local >= tier.cta_count;
  const GroupWork work(tier.cols, tier.cta_count > 0 ? tier.cta_count : 1, local, kWideBoxesPerTile);
  const int ntiles = idle ? 0 : work.ntiles;
  auto tile_box0 = [&](int j) { return work.box_begin + j * kWideBoxesPerTile; };
  auto tile_nbox = [&](int j) { return min(kWideBoxesPerTile, work.box_end - tile_box0(j)); };
  const int nkb = (p.K + kWideBK - 1) / kWideBK;
  // Paired mode: this CTA's 256-token row of the batch.
  const int tok0 = PAIR ? (int)blockIdx.y * kWideHalf : 0;

  const uint32_t full0 = sbase + L::bar_off;
  const uint32_t empty0 = full0 + S * 8;
  const uint32_t tfull = empty0 + S * 8;
  const uint32_t tempty = tfull + 8;
  uint32_t *tmem_base_slot = reinterpret_cast<uint32_t *>(smem + L::misc_off);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + L::misc_off + 4);
  const WaitCtx wc{abort_flag, p.status};

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(full0 + 8 * s, 1);
      mbar_init(empty0 + 8 * s, 1);
    }
    mbar_init(tfull, 1);
    mbar_init(tempty, kMmaEpiWarps);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(sbase + L::misc_off, kWideTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_base_slot;
  if (threadIdx.x == 0) griddep_launch_dependents();

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0 && ntiles > 0 && nkb > 0) {
      prefetch_tensormap(&tier.wmap);
      prefetch_tensormap(&p.xmap);
      const uint64_t pol_w = l2_policy_evict_first();
      const uint64_t pol_x = l2_policy_evict_last();
      uint32_t issued_mask = 0, issued_par = 0;
      const int total = ntiles * nkb;
      auto w_loads = [&](int i, uint32_t fb) {
        const int j = i / nkb, kb = i % nkb;
        const int nbox = tile_nbox(j);
        mbar_arrive_expect_tx(fb, (uint32_t)nbox * kWideWBox + L::x_stage);
        const uint32_t wdst = sbase + L::w_off + (i % S) * L::w_stage;
        for (int bx = 0; bx < nbox; ++bx)
          tma_load_2d(wdst + bx * kWideWBox, &tier.wmap, (tile_box0(j) + bx) * kBoxCols, kb * kWideBK, fb, pol_w);
      };
      auto x_load = [&](int i, uint32_t fb) {
        const uint32_t xdst = sbase + L::x_off + (i % S) * L::x_stage;
        // Rows past the batch read as zeros (tile-map bounds), so every box
        // is full.
        for (int h = 0; h < L::x_boxes; ++h)
          tma_load_2d(xdst + h * kWideXBox, &p.xmap, (i % nkb) * kWideBK, tok0 + h * kWideHalf, fb, pol_x);
      };
      // Weights do not depend on the previous kernel of the stream.
      const int pre = p.pdl ? min(total, S) : 0;
      for (int i = 0; i < pre; ++i) w_loads(i, full0 + 8 * i);
      griddep_wait();
      for (int i = 0; i < pre; ++i) {
        x_load(i, full0 + 8 * i);
        issued_mask |= 1u << i;
      }
      for (int i = pre; i < total; ++i) {
        const int s = i % S;
        const uint32_t ph = (uint32_t)((i / S) & 1);
        if (!mbar_wait<false>(empty0 + 8 * s, ph ^ 1u, wc)) break;
        const uint32_t fb = full0 + 8 * s;
        w_loads(i, fb);
        x_load(i, fb);
        issued_mask |= 1u << s;
        issued_par = (issued_par & ~(1u << s)) | (ph << s);
      }
      if (*abort_flag) {
        // Let the copies in flight land before the CTA's shared memory goes away.
        const WaitCtx drain{reinterpret_cast<volatile int *>(smem + L::misc_off + 8), p.status};
        *drain.abort = 0;
        for (int st = 0; st < S; ++st)
          if (issued_mask & (1u << st)) mbar_wait<false>(full0 + 8 * st, (issued_par >> st) & 1u, drain);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issue
    if (ntiles > 0 && nkb > 0) {
      constexpr uint32_t idesc = mma_idesc<T>(kWideHalf);
      int s = 0;
      uint32_t ph = 0;
      for (int j = 0; j < ntiles; ++j) {
        // Paired mode: a last unit of one or two boxes leaves the second
        // accumulator without weights.
        const int halves = PAIR ? (tile_nbox(j) > 2 ? 2 : 1) : 2;
        // Wait until the epilogue has read the previous tile's accumulators.
        mbar_wait<false>(tempty, ((uint32_t)j & 1u) ^ 1u, wc);
        tc_fence_after();
        for (int kb = 0; kb < nkb; ++kb) {
          const bool ok = mbar_wait<false>(full0 + 8 * s, ph, wc);
          tc_fence_after();
          if (lane == 0) {
            if (ok) {
              const uint32_t wst = sbase + L::w_off + s * L::w_stage;
              const uint32_t xst = sbase + L::x_off + s * L::x_stage;
#pragma unroll
              for (int kk = 0; kk < kWideBK / 16; ++kk) {
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                  if (h < halves) {
                    // A: MN-major SW128; 16 K rows = 2 KB; LBO = next 64-feature box, SBO = 8 rows.
                    // Paired mode: accumulator h takes the tile of boxes 2h and 2h + 1.
                    const uint64_t ad =
                        smem_desc_sw128(wst + (PAIR ? h * 2 * kWideWBox : 0u) + kk * 2048, kWideWBox, 1024);
                    // B: K-major SW128; 16 K = 32 B inside the 128-byte span; SBO = 8 rows.
                    // Unpaired: accumulator h takes token half h.
                    const uint64_t bd = smem_desc_sw128(xst + (PAIR ? 0u : h * kWideXBox) + kk * 32, 16, 1024);
                    tc_mma_f16(tmem_base + (uint32_t)(h * kWideHalf), ad, bd, idesc,
                               (kb > 0 || kk > 0) ? 1u : 0u);
                  }
                }
              }
            }
            tc_commit(empty0 + 8 * s);  // frees the stage once these MMAs have read it
          }
          __syncwarp();
          if (++s == S) {
            s = 0;
            ph ^= 1u;
          }
        }
        if (lane == 0) tc_commit(tfull);
        __syncwarp();
      }
      // Before TMEM is freed, the last MMAs must have finished, also when the
      // epilogue gave up waiting for them.
      const WaitCtx last{reinterpret_cast<volatile int *>(smem + L::misc_off + 12), p.status};
      if (lane == 0) {
        *last.abort = 0;
        mbar_wait<false>(tfull, (uint32_t)(ntiles - 1) & 1u, last);
      }
      __syncwarp();
    }
  } else {
    // ------------------------------------------------------------- epilogue
    griddep_wait();  // y may still be read by the previous kernel of the stream
    const int qd = warp & 3;                 // TMEM lane quadrant of this warp
    const int f = qd * 32 + lane;            // feature within the 128-feature tile
    const uint32_t lane_addr = (uint32_t)(qd * 32) << 16;
    if (nkb > 0) {
      for (int j = 0; j < ntiles; ++j) {
        mbar_wait<false>(tfull, (uint32_t)j & 1u, wc);
        tc_fence_after();
        // Unpaired: one 128-feature tile, token t in accumulator column t (both
        // accumulators).  Paired: accumulator h holds features [128h, 128h + 128)
        // of the unit for the CTA's token row.
        const int nfeat = tile_nbox(j) * kBoxCols;
        const int nacc = PAIR ? (tile_nbox(j) > 2 ? 2 : 1) : 1;
        const int ntok_here = PAIR ? min(kWideHalf, p.ntok - tok0) : p.ntok;  // warp-uniform
        for (int h = 0; h < nacc; ++h) {
          const int fo = (PAIR ? h * kMmaBM : 0) + f;
          const int col = tile_box0(j) * kBoxCols + fo;
          const bool col_ok = fo < nfeat && col < tier.cols;
          uint16_t *ycol = reinterpret_cast<uint16_t *>(p.y) + (long long)tok0 * p.ldy + tier.col_offset + col;
          const uint32_t acc = PAIR ? (uint32_t)(h * kWideHalf) : 0u;
#pragma unroll 1
          for (int c0 = 0; c0 < ntok_here; c0 += 32) {
            float v[32];
            tmem_ld32(tmem_base + lane_addr + acc + (uint32_t)c0, v);
            if (col_ok) {
#pragma unroll
              for (int t = 0; t < 32; ++t)
                if (c0 + t < ntok_here) ycol[(long long)(c0 + t) * p.ldy] = Elem<T>::from_float(v[t]);
            }
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(tempty);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, kWideTmemCols);
}

}  // namespace

size_t linear_wide_smem_bytes(bool pair) { return pair ? WideLayout<true>::bytes : WideLayout<false>::bytes; }

int linear_wide_k_rows() { return kWideBK; }

cudaError_t launch_linear_wide(const LinearParams &p, int dtype, int grid, size_t smem, cudaStream_t stream,
                               bool pair) {
  if (dtype == DAK_DTYPE_F16)
    return pair ? launch_linear_kernel(linear_wide_kernel<__half, true>, p, grid, kMmaThreads, 1, smem, stream, nullptr)
                : launch_linear_kernel(linear_wide_kernel<__half, false>, p, grid, kMmaThreads, 1, smem, stream,
                                       nullptr);
  if (dtype == DAK_DTYPE_BF16)
    return pair ? launch_linear_kernel(linear_wide_kernel<__nv_bfloat16, true>, p, grid, kMmaThreads, 1, smem,
                                       stream, nullptr)
                : launch_linear_kernel(linear_wide_kernel<__nv_bfloat16, false>, p, grid, kMmaThreads, 1, smem,
                                       stream, nullptr);
  return cudaErrorInvalidValue;
}

}  // namespace dak
