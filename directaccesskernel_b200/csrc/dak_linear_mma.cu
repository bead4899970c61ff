// dak_linear_mma.cu - split-tier offloaded linear on the 5th-generation tensor
// cores (tcgen05.mma kind::f16, FP32 accumulators in TMEM), for batched decode
// and prefill (from 3 tokens under the automatic path choice, 256 per launch).
//
// Replaces the reference's wgmma kernels `gemv_multicast`,
// `gemv_horizontal_multicast` and their `_prefill` variants
// (include/task/gemv_multicast.cuh:185-914), which multicast 64x64 weight
// tiles to a 2-CTA cluster and accumulate in FP16.  Here the GEMM is "swap-AB":
// 128 output features form the UMMA M dimension and the tokens the UMMA N
// dimension (16..256), so one CTA applies each weight tile to all tokens and no
// weight byte is fetched twice - no multicast is needed or used.
//
// Roles (192 threads): warp 0 issues TMA loads (two 64-feature x 128-row
// weight boxes with 128-byte swizzle, MN-major, plus two 64-wide activation
// boxes, K-major, per stage); warp 1 owns TMEM and issues the MMAs from one
// lane; warps 2..5 read the accumulators back with tcgen05.ld (each warp its
// TMEM lane quadrant) and write the 16-bit output.  Each group of `ksplit`
// CTAs owns a contiguous, evenly sized range of 64-feature boxes, walked as
// 128-feature tiles; the CTAs of a group split K and reduce-scatter through
// DSMEM: each owns 128/ksplit features of the tile, receives the other CTAs'
// partials for them in its own shared memory and writes them out.  Launched
// with programmatic stream serialization, the producer fills the ring with
// weights before waiting for the previous kernel of the stream.
#include "dak_common.cuh"
#include "dak_host.h"
#include "dak_linear.cuh"
#include "dak_tcgen05.cuh"

#include <type_traits>

namespace dak {

namespace {

constexpr uint32_t kMmaBoxBytes = kBoxCols * kMmaBK * 2;       // 16 KB (64 x 128)
constexpr uint32_t kMmaWStageBytes = 2 * kMmaBoxBytes;         // 32 KB (128 x 128)
constexpr int kMmaBoxesPerTile = kMmaBM / kBoxCols;            // 2
constexpr int kMmaMaxKsplit = 4;
constexpr int kMmaMaxStages = 8;
constexpr uint32_t kSmemPerBlock = 227 * 1024;

// Shared-memory layout; the pipeline depth is chosen at launch so that the
// stages and the split-K receive buffer fit in one SM's shared memory.
template <int NTOKP>
struct MmaLayout {
  // Activations: two K-major 128-byte-swizzled boxes of NTOKP rows x 64 k.
  static constexpr uint32_t x_box_bytes = NTOKP * 128;
  static constexpr uint32_t x_stage_bytes = 2 * x_box_bytes;
  static constexpr uint32_t red_row = NTOKP + 4;  // floats per feature row (padded)
  int stages;
  uint32_t w_off, x_off, bar_off, misc_off, red_off;
  __host__ __device__ explicit MmaLayout(int s) : stages(s) {
    w_off = 0;
    x_off = w_off + (uint32_t)s * kMmaWStageBytes;
    bar_off = x_off + (uint32_t)s * x_stage_bytes;
    // full[S], empty[S], tmem_full[2], tmem_empty[2], red_full, red_free
    misc_off = bar_off + (uint32_t)(2 * s + 6) * 8;  // tmem base slot, abort flags
    red_off = (misc_off + 16 + 15) & ~15u;
  }
  __host__ __device__ static constexpr uint32_t red_floats(int ks) {
    return ks > 1 ? (uint32_t)(ks - 1) * (uint32_t)(kMmaBM / ks) * red_row : 0u;
  }
  __host__ __device__ uint32_t bytes(int ks) const { return red_off + red_floats(ks) * 4 + 1024; }
  __host__ __device__ static constexpr uint32_t tmem_cols() {
    return (2 * NTOKP <= 32) ? 32 : (2 * NTOKP <= 64) ? 64 : (2 * NTOKP <= 128) ? 128
           : (2 * NTOKP <= 256) ? 256 : 512;
  }
};

// System-scope release store / acquire load of a 32-bit flag in (possibly peer)
// global memory, for the fused all-reduce.
__device__ __forceinline__ void st_release_sys(uint32_t *p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
// Sum over all ranks of a 32-bit float at a multicast address (reduced in the switch).
__device__ __forceinline__ float multimem_ld_reduce_add(const float *p) {
  float v;
  // No memory clobber: a batch of these is issued before any result is used;
  // volatile keeps them after the barrier that follows the flag wait.
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.f32 %0, [%1];" : "=f"(v) : "l"(p));
  return v;
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t *p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

template <typename T, int NTOKP, bool AR>
__global__ void __launch_bounds__(kMmaThreads, 1)
    linear_mma_kernel(const __grid_constant__ LinearParams p) {
  const MmaLayout<NTOKP> L(p.stages);
  const int S = L.stages;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_u32 = smem_u32(smem_raw);
  uint8_t *smem = smem_raw + (((raw_u32 + 1023u) & ~1023u) - raw_u32);
  const uint32_t sbase = smem_u32(smem);

  const int warp = warp_id();
  const int lane = lane_id();

  const int ti = (p.tier[1].cta_count > 0 && (int)blockIdx.x >= p.tier[1].cta_begin) ? 1 : 0;
  const LinearTier &tier = p.tier[ti];
  const int local = (int)blockIdx.x - tier.cta_begin;
  const int ks = tier.ksplit;
  const int groups = tier.cta_count / ks;
  const int g = local / ks;
  const int r = local - g * ks;
  // CTAs that only pad the tier to a whole number of clusters do no work.
  const bool idle = local >= tier.cta_count;
  const GroupWork work(tier.cols, groups > 0 ? groups : 1, g, kMmaBoxesPerTile);
  const int ntiles = idle ? 0 : work.ntiles;
  auto tile_box0 = [&](int j) { return work.box_begin + j * kMmaBoxesPerTile; };
  auto tile_nbox = [&](int j) { return min(kMmaBoxesPerTile, work.box_end - tile_box0(j)); };
  const int nkb = (p.K + kMmaBK - 1) / kMmaBK;
  const int kb0 = (int)((long long)r * nkb / ks);
  const int kb1 = (int)((long long)(r + 1) * nkb / ks);
  const int feat_per_owner = kMmaBM / ks;  // features each CTA of the group writes
  // Token slice of this grid row: tokens [tok0, tok0 + NTOKP) of every tile
  // (grid rows > 1 only without the fused all-reduce).
  const int tok0 = AR ? 0 : (int)blockIdx.y * NTOKP;

  const uint32_t full0 = sbase + L.bar_off;
  const uint32_t empty0 = full0 + S * 8;
  const uint32_t tfull0 = empty0 + S * 8;
  const uint32_t tempty0 = tfull0 + 16;
  const uint32_t red_full = tempty0 + 16;
  const uint32_t red_free = red_full + 8;
  uint32_t *tmem_base_slot = reinterpret_cast<uint32_t *>(smem + L.misc_off);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + L.misc_off + 4);
  float *red = reinterpret_cast<float *>(smem + L.red_off);
  const WaitCtx wc{abort_flag, p.status};

  // Owners receive (ks-1) senders x (4/ks) warps x 32 lanes arrivals per round;
  // senders get one arrival from lane 0 of every owner warp of the other ranks.
  const uint32_t red_full_count = ks > 1 ? (uint32_t)((ks - 1) * (kMmaEpiWarps / ks) * 32) : 1u;
  const uint32_t red_free_count = ks > 1 ? (uint32_t)((ks - 1) * (kMmaEpiWarps / ks)) : 1u;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(full0 + 8 * s, 1);
      mbar_init(empty0 + 8 * s, 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(tfull0 + 8 * a, 1);
      mbar_init(tempty0 + 8 * a, kMmaEpiWarps);
    }
    mbar_init(red_full, red_full_count);
    mbar_init(red_free, red_free_count);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(sbase + L.misc_off, L.tmem_cols());
    tmem_relinquish();
  }
  tc_fence_before();
  cluster_sync_all();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_base_slot;
  // The next layer may be scheduled now: it only prefetches its own weights
  // until this grid has completed.
  if (threadIdx.x == 0) griddep_launch_dependents();

  bool sent_remote = false;  // this thread's last tile ended with writes to a peer's shared memory
  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0 && ntiles > 0 && kb1 > kb0) {
      prefetch_tensormap(&tier.wmap);
      prefetch_tensormap(&p.xmap);
      const uint64_t pol_w = l2_policy_evict_first();
      const uint64_t pol_x = l2_policy_evict_last();
      uint32_t issued_mask = 0, issued_par = 0;
      // Work items in order: tiles g, g+groups, ... each over k blocks [kb0, kb1).
      const int nk = kb1 - kb0;
      const int total = ntiles * nk;
      auto w_loads = [&](int i, uint32_t fb) {
        const int j = i / nk, kb = kb0 + i % nk;
        const int nbox = tile_nbox(j);
        mbar_arrive_expect_tx(fb, (uint32_t)nbox * kMmaBoxBytes + L.x_stage_bytes);
        const uint32_t wdst = sbase + L.w_off + (i % S) * kMmaWStageBytes;
        for (int bx = 0; bx < nbox; ++bx)
          tma_load_2d(wdst + bx * kMmaBoxBytes, &tier.wmap, (tile_box0(j) + bx) * kBoxCols, kb * kMmaBK, fb, pol_w);
      };
      auto x_load = [&](int i, uint32_t fb) {
        const uint32_t xdst = sbase + L.x_off + (i % S) * L.x_stage_bytes;
        for (int h = 0; h < 2; ++h)
          tma_load_2d(xdst + h * L.x_box_bytes, &p.xmap, (kb0 + i % nk) * kMmaBK + h * 64, tok0, fb, pol_x);
      };
      // Weights do not depend on the previous kernel of the stream: fill the
      // ring with them first, then wait for that kernel before touching x.
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
        const WaitCtx drain{reinterpret_cast<volatile int *>(smem + L.misc_off + 8), p.status};
        *drain.abort = 0;
        for (int st = 0; st < S; ++st)
          if (issued_mask & (1u << st)) mbar_wait<false>(full0 + 8 * st, (issued_par >> st) & 1u, drain);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issue
    if (ntiles > 0 && kb1 > kb0) {
      constexpr uint32_t idesc = mma_idesc<T>(NTOKP);
      int s = 0;
      uint32_t ph = 0;
      int n = 0;
      for (int j = 0; j < ntiles; ++j, ++n) {
        const int ab = n & 1;
        const uint32_t use = (uint32_t)(n >> 1);
        // Wait until the epilogue drained this accumulator buffer.
        mbar_wait<false>(tempty0 + 8 * ab, (use & 1u) ^ 1u, wc);
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(ab * NTOKP);
        for (int kb = kb0; kb < kb1; ++kb) {
          const bool ok = mbar_wait<false>(full0 + 8 * s, ph, wc);
          tc_fence_after();
          if (lane == 0) {
            if (ok) {
              const uint32_t wst = sbase + L.w_off + s * kMmaWStageBytes;
              const uint32_t xst = sbase + L.x_off + s * L.x_stage_bytes;
#pragma unroll
              for (int kk = 0; kk < kMmaBK / 16; ++kk) {
                // A: MN-major SW128; 16 K rows = 2 KB; LBO = next 64-feature box, SBO = 8 rows.
                const uint64_t ad = smem_desc_sw128(wst + kk * 2048, kMmaBoxBytes, 1024);
                // B: K-major SW128; 64 K per box, 16 K = 32 B inside the swizzle span; SBO = 8 rows.
                const uint64_t bd = smem_desc_sw128(xst + (kk >> 2) * L.x_box_bytes + (kk & 3) * 32, 16, 1024);
                tc_mma_f16(d_tmem, ad, bd, idesc, (kb > kb0 || kk > 0) ? 1u : 0u);
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
        if (lane == 0) tc_commit(tfull0 + 8 * ab);
        __syncwarp();
      }
    }
  } else {
    // ------------------------------------------------------------- epilogue
    griddep_wait();  // y may still be read by the previous kernel of the stream
    const int qd = warp & 3;                 // TMEM lane quadrant of this warp
    const int f = qd * 32 + lane;            // feature within the 128-feature tile
    const int owner = (qd * 32) / feat_per_owner;  // rank of the group that writes f
    // Accumulator columns moved per tcgen05.ld; never more than the tile has.
    constexpr int kChunkCols = NTOKP < 32 ? NTOKP : 32;
    const uint32_t my_rank = cluster_ctarank();
    const uint32_t lane_addr = (uint32_t)(qd * 32) << 16;
    int n = 0;
    int nred = 0;
    // Fused all-reduce: this call's epoch, and where this rank's partial goes in
    // every rank's receive buffer (slot `rank` of parity epoch & 1).
    const uint32_t ar_epoch = AR ? (uint32_t)(*reinterpret_cast<volatile int *>(p.ar.epoch) + 1) : 0u;
    const long long ar_slot =
        !AR ? 0 : p.ar.mc ? (long long)(ar_epoch & 1u) * p.ar.slot_elems
                          : ((long long)(ar_epoch & 1u) * p.ar.world + p.ar.rank) * p.ar.slot_elems;
    if (kb1 > kb0) {
      for (int j = 0; j < ntiles; ++j, ++n) {
        const int ab = n & 1;
        const uint32_t use = (uint32_t)(n >> 1);
        mbar_wait<false>(tfull0 + 8 * ab, use & 1u, wc);
        tc_fence_after();
        const uint32_t acc_addr = tmem_base + lane_addr + (uint32_t)(ab * NTOKP);
        const int col = tile_box0(j) * kBoxCols + f;
        const bool col_ok = f < tile_nbox(j) * kBoxCols && col < tier.cols;
        T *ycol = reinterpret_cast<T *>(p.y) + (long long)tok0 * p.ldy + tier.col_offset + col;

        if (ks == 1 || owner == r) {
          if (ks > 1) mbar_wait<true>(red_full, (uint32_t)(nred & 1), wc);
          const int fl = f - owner * feat_per_owner;
#pragma unroll 1
          for (int c0 = 0; c0 < NTOKP; c0 += kChunkCols) {
            float v[kChunkCols];
            tmem_ld_chunk<kChunkCols>(acc_addr + (uint32_t)c0, v);
            if (ks > 1) {
              for (int m = 0; m < ks - 1; ++m) {
                const float *src = red + ((size_t)m * feat_per_owner + fl) * L.red_row + c0;
#pragma unroll
                for (int j = 0; j < kChunkCols; j += 4) {
                  const float4 a = *reinterpret_cast<const float4 *>(src + j);
                  v[j] += a.x; v[j + 1] += a.y; v[j + 2] += a.z; v[j + 3] += a.w;
                }
              }
            }
            if (!AR && p.glu) {
              // Gated output: gate and up rows alternate in blocks of 16
              // features, so lane l < 16 holds gate feature g of this block
              // and lane l + 16 the matching up feature; y column
              // (c / 32) * 16 + c % 16 gets silu(gate) * up, rounded once.
              const int c = tier.col_offset + col;
              uint16_t *yg = reinterpret_cast<uint16_t *>(p.y) + (long long)tok0 * p.ldy + (c >> 5) * 16 + (c & 15);
#pragma unroll
              for (int j = 0; j < kChunkCols; ++j) {
                const float up = __shfl_xor_sync(0xffffffffu, v[j], 16);
                if (col_ok && lane < 16 && tok0 + c0 + j < p.ntok)
                  yg[(long long)(c0 + j) * p.ldy] = Elem<T>::from_float(v[j] / (1.f + expf(-v[j])) * up);
              }
            } else if (col_ok) {
              if (AR) {
                const long long base = ar_slot + tier.col_offset + col;
                if (p.ar.mc) {
#pragma unroll
                  for (int j = 0; j < kChunkCols; ++j)
                    if (c0 + j < p.ntok) p.ar.own[base + (long long)(c0 + j) * p.ldy] = v[j];
                } else {
#pragma unroll
                  for (int j = 0; j < kChunkCols; ++j)
                    if (c0 + j < p.ntok) {
                      const uint16_t h = Elem<T>::from_float(v[j]);
                      for (int rk = 0; rk < p.ar.world; ++rk)
                        p.ar.buf[rk][base + (long long)(c0 + j) * p.ldy] = h;
                    }
                }
              } else {
#pragma unroll
                for (int j = 0; j < kChunkCols; ++j)
                  if (tok0 + c0 + j < p.ntok)
                    reinterpret_cast<uint16_t *>(ycol)[(long long)(c0 + j) * p.ldy] =
                        Elem<T>::from_float(v[j]);
              }
            }
          }
          if (ks > 1) {
            __syncwarp();
            // Senders wait for this before sending their next partial; after
            // the last tile there is none, and a sender may already have left.
            if (lane == 0 && j + 1 < ntiles)
              for (int m = 0; m < ks; ++m)
                if (m != r) mbar_arrive_remote(mapa_shared(red_free, my_rank - r + m));
          }
        } else {
          // Sender: push this warp's partial to the owner of its features.
          if (nred > 0) mbar_wait<true>(red_free, (uint32_t)((nred - 1) & 1), wc);
          const int slot = r < owner ? r : r - 1;
          const int fl = f - owner * feat_per_owner;
          const uint32_t owner_rank = my_rank - r + owner;
          const uint32_t dst_base = mapa_shared(
              smem_u32(red + ((size_t)slot * feat_per_owner + fl) * L.red_row), owner_rank);
#pragma unroll 1
          for (int c0 = 0; c0 < NTOKP; c0 += kChunkCols) {
            float v[kChunkCols];
            tmem_ld_chunk<kChunkCols>(acc_addr + (uint32_t)c0, v);
#pragma unroll
            for (int j = 0; j < kChunkCols; j += 4)
              st_cluster_v4(dst_base + (uint32_t)(c0 + j) * 4, v[j], v[j + 1], v[j + 2], v[j + 3]);
          }
          mbar_arrive_remote(mapa_shared(red_full, owner_rank));
          sent_remote = true;
        }
        if (ks > 1) ++nred;
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(tempty0 + 8 * ab);
      }
    }
    if (AR && p.ar.publish_only) {
      // ---- publish only: the partials stay in this rank's buffer; the last
      // CTA to finish tells every rank that call e is complete, and the
      // consumer kernel (dak_rmsnorm_allreduce) reads the sum over ranks.
      __threadfence_system();
      named_sync(2, kMmaEpiWarps * 32);
      if (warp == 2 && lane == 0) {
        __threadfence_system();
        if (atomicAdd(p.ar.done, 1) == (int)gridDim.x - 1) {
          *p.ar.done = 0;
          __threadfence_system();
          for (int rk = 0; rk < p.ar.world; ++rk) st_release_sys(p.ar.flags[rk] + p.ar.rank, ar_epoch);
          atomicExch(p.ar.epoch, (int)ar_epoch);
        }
      }
      __syncwarp();
    } else if (AR) {
      // ---- fused all-reduce: publish, wait for every rank's same CTA, sum
      const int W = p.ar.world, me = p.ar.rank, c = (int)blockIdx.x;
      volatile int *ar_fail = abort_flag + 2;
      __threadfence_system();
      named_sync(2, kMmaEpiWarps * 32);
      if (warp == 2 && lane == 0) {
        *ar_fail = 0;
        for (int rk = 0; rk < W; ++rk) st_release_sys(p.ar.flags[rk] + (long long)c * W + me, ar_epoch);
        const unsigned long long t0 = globaltimer();
        for (int rk = 0; rk < W && !*ar_fail; ++rk)
          while ((int)(ld_acquire_sys(p.ar.flags[me] + (long long)c * W + rk) - ar_epoch) < 0) {
            if (globaltimer() - t0 > (unsigned long long)p.ar.timeout_ns) {
              atomicCAS(p.status, 0, DAK_ERR_TIMEOUT);
              *ar_fail = 1;
              break;
            }
          }
      }
      __syncwarp();
      named_sync(2, kMmaEpiWarps * 32);
      if (!*ar_fail && kb1 > kb0) {
        const uint16_t *rb = p.ar.mc ? nullptr : p.ar.buf[me] + (long long)(ar_epoch & 1u) * W * p.ar.slot_elems;
        const float *mb = p.ar.mc ? p.ar.mc + (long long)(ar_epoch & 1u) * p.ar.slot_elems : nullptr;
        // All 128 epilogue threads share the CTA's owned (row, feature) elements,
        // feature fastest, and issue kBatch independent reductions before using
        // any result, so the latency of the reads overlaps.
        constexpr int kBatch = 8;
        const int et = (warp - 2) * 32 + lane;
        for (int j = 0; j < ntiles; ++j) {
          const int base_col = tile_box0(j) * kBoxCols;
          const int f_lo = ks == 1 ? 0 : r * feat_per_owner;
          int f_hi = ks == 1 ? kMmaBM : f_lo + feat_per_owner;
          f_hi = min(f_hi, min(tile_nbox(j) * kBoxCols, tier.cols - base_col));
          const int ncols = f_hi - f_lo;
          if (ncols <= 0) continue;
          const long long n = (long long)ncols * p.ntok;
          const long long cbase = tier.col_offset + base_col + f_lo;
          for (long long e0 = et; e0 < n; e0 += (long long)kMmaEpiWarps * 32 * kBatch) {
            long long idx[kBatch];
            float acc[kBatch];
#pragma unroll
            for (int u = 0; u < kBatch; ++u) {
              const long long e = e0 + (long long)u * kMmaEpiWarps * 32;
              const long long row = e < n ? e / ncols : 0;
              idx[u] = e < n ? row * p.ldy + cbase + (e - row * ncols) : -1;
            }
            if (mb) {
#pragma unroll
              for (int u = 0; u < kBatch; ++u) acc[u] = idx[u] >= 0 ? multimem_ld_reduce_add(mb + idx[u]) : 0.f;
            } else {
#pragma unroll
              for (int u = 0; u < kBatch; ++u) {
                acc[u] = 0.f;
                if (idx[u] >= 0)
                  for (int rk = 0; rk < W; ++rk)
                    acc[u] += Elem<T>::to_float(rb[(long long)rk * p.ar.slot_elems + idx[u]]);
              }
            }
#pragma unroll
            for (int u = 0; u < kBatch; ++u)
              if (idx[u] >= 0) reinterpret_cast<uint16_t *>(p.y)[idx[u]] = Elem<T>::from_float(acc[u]);
          }
        }
      }
      named_sync(2, kMmaEpiWarps * 32);
      if (warp == 2 && lane == 0) {
        __threadfence();
        if (atomicAdd(p.ar.done, 1) == (int)gridDim.x - 1) {
          *p.ar.done = 0;
          __threadfence();
          atomicExch(p.ar.epoch, (int)ar_epoch);
        }
      }
      __syncwarp();
    }
  }

  // No CTA leaves while a peer may still touch its shared memory (see
  // cluster_exit_sync): owners waited for every partial sent to them and send
  // no release after the last tile, so only senders need release semantics;
  // the output stores need none.
  tc_fence_before();
  cluster_exit_sync(sent_remote);
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, L.tmem_cols());
}

template <typename T>
cudaError_t launch_dtype(const LinearParams &p, int ntokp, int grid, int cluster, size_t smem,
                         cudaStream_t stream, int *mc) {
  // The fused all-reduce is a separate instantiation, so the plain kernel
  // carries none of its code or registers.
#define DAK_MMA_CASE(N)                                                                                  \
  case N:                                                                                                \
    return p.ar_on ? launch_linear_kernel(linear_mma_kernel<T, N, true>, p, grid, kMmaThreads, cluster, smem, \
                                          stream, mc)                                                    \
                   : launch_linear_kernel(linear_mma_kernel<T, N, false>, p, grid, kMmaThreads, cluster, smem, \
                                          stream, mc);
  switch (ntokp) {
    DAK_MMA_CASE(16)
    DAK_MMA_CASE(32)
    DAK_MMA_CASE(64)
    DAK_MMA_CASE(128)
    DAK_MMA_CASE(256)
    default: return cudaErrorInvalidValue;
  }
#undef DAK_MMA_CASE
}

template <int NTOKP>
int stages_for(int ks) {
  int st = kMmaMaxStages;
  while (st > 2 && MmaLayout<NTOKP>(st).bytes(ks) > kSmemPerBlock) --st;
  return st;
}

template <int NTOKP>
size_t smem_for(int ks) {
  return MmaLayout<NTOKP>(stages_for<NTOKP>(ks)).bytes(ks);
}

}  // namespace

int linear_mma_stages(int ntokp, int ksplit) {
  switch (ntokp) {
    case 16: return stages_for<16>(ksplit);
    case 32: return stages_for<32>(ksplit);
    case 64: return stages_for<64>(ksplit);
    case 128: return stages_for<128>(ksplit);
    case 256: return stages_for<256>(ksplit);
    default: return 0;
  }
}

// `red_slots` is the largest ksplit of the launch minus one.
size_t linear_mma_smem_bytes(int ntokp, int red_slots) {
  const int ks = red_slots + 1;
  if (ks > kMmaMaxKsplit || (ks & (ks - 1)) != 0) return 0;
  switch (ntokp) {
    case 16: return smem_for<16>(ks);
    case 32: return smem_for<32>(ks);
    case 64: return smem_for<64>(ks);
    case 128: return smem_for<128>(ks);
    case 256: return smem_for<256>(ks);
    default: return 0;
  }
}

cudaError_t launch_linear_mma(const LinearParams &p, int ntokp, int dtype, int grid, int cluster,
                              size_t smem, cudaStream_t stream, int *max_clusters) {
  if (dtype == DAK_DTYPE_F16) return launch_dtype<__half>(p, ntokp, grid, cluster, smem, stream, max_clusters);
  if (dtype == DAK_DTYPE_BF16)
    return launch_dtype<__nv_bfloat16>(p, ntokp, grid, cluster, smem, stream, max_clusters);
  return cudaErrorInvalidValue;
}

}  // namespace dak
