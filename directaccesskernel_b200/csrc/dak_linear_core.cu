// dak_linear_core.cu - split-tier offloaded linear for decode (ntok <= 8),
// CUDA-core FP32 FMAs with warp-shuffle reductions.
//
// Replaces the reference's `gemv` / `gemv_horizontal` (include/task/gemv.cuh:
// 267-452), which feed wgmma with FP16 accumulation on sm_90a.  Here:
//   * one CTA = 1 producer warp + 8 consumer warps;
//   * the producer streams 128-feature x 128-row weight stages (2 TMA boxes of
//     64 x 128, 128-byte swizzle) and the matching activation slice through an
//     mbarrier ring sized to the shared memory; the host tier's CTAs read
//     pinned host memory over the host link, the device tier's CTAs read HBM,
//     in the same launch;
//   * each group of `ksplit` CTAs owns a contiguous, evenly sized range of
//     64-feature boxes (so no group has more than one box above the average)
//     and walks it as tiles of up to 2 boxes; the CTAs of the group split K;
//   * consumer warp w = (kq, hc, b) owns 32 features (box b, 64-byte half hc)
//     over the row half kq of every stage; lane (q, ro) reads 16 bytes of rows
//     ro, ro+8, ... and keeps FP32 partial sums for 8 features x NTOK tokens; a
//     3-step xor shuffle sums the 8 row groups (the warp-shuffle reduction) and
//     the two row halves meet in shared memory;
//   * the K-split partials of a tile are summed in the leader CTA's shared
//     memory through DSMEM stores and remote mbarrier arrivals (no global
//     scratch, no atomics);
//   * the result is cast to 16-bit once and written with plain stores, so the
//     output needs no zero fill (the reference reduce-adds into a zeroed C);
//   * launched with programmatic stream serialization, the producer fills the
//     ring with weights before waiting for the previous kernel of the stream.
#include "dak_common.cuh"
#include "dak_host.h"
#include "dak_linear.cuh"

namespace dak {

namespace {

constexpr uint32_t kCoreWStageBytes = kCoreBN * kCoreBK * 2;   // 32 KB
constexpr uint32_t kCoreBoxBytes = kBoxCols * kCoreBK * 2;     // 16 KB
constexpr uint32_t kCoreSmemBudget = 227 * 1024;
constexpr int kCoreRowHalf = kCoreBK / 2;                      // rows per consumer row half
constexpr int kCoreReduceWarps = kCoreConsumerWarps / 2;       // row-half-0 warps own the outputs

template <int NTOK>
struct CoreLayout {
  static constexpr uint32_t x_stage_bytes = NTOK * kCoreBK * 2;
  static constexpr uint32_t x_stage_stride = (x_stage_bytes + 127) & ~127u;
  static constexpr uint32_t red_slot_floats = NTOK * kCoreBN;
  static constexpr uint32_t comb_floats = NTOK * kCoreBN;  // one row-half hand-off buffer
  int stages;
  uint32_t w_off, x_off, bar_off, flag_off, comb_off, red_off;
  __host__ __device__ explicit CoreLayout(int s) : stages(s) {
    w_off = 0;
    x_off = w_off + (uint32_t)s * kCoreWStageBytes;
    bar_off = x_off + (uint32_t)s * x_stage_stride;
    flag_off = bar_off + (uint32_t)(2 * s + 2) * 8;  // full[S], empty[S], red_full, red_free
    comb_off = (flag_off + 16 + 15) & ~15u;
    red_off = comb_off + 2 * comb_floats * 4;        // double-buffered by tile parity
  }
  __host__ __device__ uint32_t bytes(int red_slots) const {
    return red_off + (uint32_t)red_slots * red_slot_floats * 4 + 1024;  // +1024: base alignment
  }
  static int stages_for(int red_slots) {
    int s = kCoreStages;
    while (s > 2 && CoreLayout(s).bytes(red_slots) > kCoreSmemBudget) --s;
    return s;
  }
};

template <typename T, int NTOK>
__global__ void __launch_bounds__(kCoreThreads, 1)
    linear_core_kernel(const __grid_constant__ LinearParams p) {
  const CoreLayout<NTOK> L(p.stages);
  const int S = L.stages;
  extern __shared__ uint8_t smem_raw[];
  // 128-byte-swizzled TMA destinations want 1024-byte alignment.
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
  const GroupWork work(tier.cols, groups > 0 ? groups : 1, g, kCoreBoxes);
  const int ntiles = idle ? 0 : work.ntiles;
  const int nkb = (p.K + kCoreBK - 1) / kCoreBK;
  const int kb0 = (int)((long long)r * nkb / ks);
  const int kb1 = (int)((long long)(r + 1) * nkb / ks);
  auto tile_box0 = [&](int j) { return work.box_begin + j * kCoreBoxes; };
  auto tile_nbox = [&](int j) { return min(kCoreBoxes, work.box_end - tile_box0(j)); };

  const uint32_t full0 = sbase + L.bar_off;
  const uint32_t empty0 = full0 + S * 8;
  const uint32_t red_full = empty0 + S * 8;
  const uint32_t red_free = red_full + 8;
  volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + L.flag_off);
  float *red = reinterpret_cast<float *>(smem + L.red_off);
  const WaitCtx wc{abort_flag, p.status};

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(full0 + 8 * s, 1);
      mbar_init(empty0 + 8 * s, kCoreConsumerWarps);
    }
    mbar_init(red_full, (uint32_t)(ks > 1 ? (ks - 1) * kCoreReduceWarps * 32 : 1));
    mbar_init(red_free, kCoreReduceWarps);
    *abort_flag = 0;
    fence_mbar_init();
  }
  // Peers arrive on these barriers, so the whole cluster waits for the inits.
  cluster_sync_all();
  // The next layer may be scheduled now: it only prefetches its own weights
  // until this grid has completed.
  if (threadIdx.x == 0) griddep_launch_dependents();

  bool sent_remote = false;  // this thread's last tile ended with writes to a peer's shared memory
  if (warp == kCoreConsumerWarps) {
    // ------------------------------------------------------------ producer
    if (lane == 0 && ntiles > 0 && kb1 > kb0) {
      prefetch_tensormap(&tier.wmap);
      prefetch_tensormap(&p.xmap);
      const uint64_t pol_w = l2_policy_evict_first();
      const uint64_t pol_x = l2_policy_evict_last();
      uint32_t issued_mask = 0, issued_par = 0;  // last issued phase per stage
      // Work items in order: the group's tiles, each over k blocks [kb0, kb1).
      const int nk = kb1 - kb0;
      const int total = ntiles * nk;
      auto w_loads = [&](int i, uint32_t fb) {
        const int j = i / nk, kb = kb0 + i % nk;
        const int nbox = tile_nbox(j);
        mbar_arrive_expect_tx(fb, (uint32_t)nbox * kCoreBoxBytes + L.x_stage_bytes);
        const uint32_t wdst = sbase + L.w_off + (i % S) * kCoreWStageBytes;
        for (int bx = 0; bx < nbox; ++bx)
          tma_load_2d(wdst + bx * kCoreBoxBytes, &tier.wmap, (tile_box0(j) + bx) * kBoxCols, kb * kCoreBK, fb,
                      pol_w);
      };
      auto x_load = [&](int i, uint32_t fb) {
        tma_load_2d(sbase + L.x_off + (i % S) * L.x_stage_stride, &p.xmap, (kb0 + i % nk) * kCoreBK, 0, fb,
                    pol_x);
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
        // Let the copies already in flight land before the CTA can exit.
        const WaitCtx drain{reinterpret_cast<volatile int *>(smem + L.flag_off + 4), p.status};
        *drain.abort = 0;
        for (int st = 0; st < S; ++st)
          if (issued_mask & (1u << st)) mbar_wait<false>(full0 + 8 * st, (issued_par >> st) & 1u, drain);
      }
    }
    __syncwarp();
  } else {
    // ----------------------------------------------------------- consumers
    griddep_wait();  // y may still be read by the previous kernel of the stream
    const int b = warp & 1;            // TMA box (64 features) of this warp
    const int hc = (warp >> 1) & 1;    // 64-byte half of the box's 128-byte rows
    const int kq = warp >> 2;          // row half of every stage
    const int q = lane & 3;            // 16-byte chunk within the warp's 64 bytes
    // Row offset 0..7 inside each 8-row group.  The 8 lanes of one shared-memory
    // phase read rows ro and ro ^ 4, whose swizzled chunks fill complementary
    // halves of the 32 banks, so the weight reads are conflict free.
    const int ro = ((lane >> 3) & 3) | (((lane >> 2) & 1) << 2);
    const int c = hc * 4 + q;          // logical 16-byte chunk in the 128-byte row
    const uint32_t chunk_off = (uint32_t)((c ^ ro) << 4);  // 128-byte swizzle: chunk ^ (row & 7)
    const int row0 = kq * kCoreRowHalf;
    float *comb = reinterpret_cast<float *>(smem + L.comb_off);
    const uint32_t my_rank = cluster_ctarank();
    int nred = 0;
    int item = 0;

    for (int j = 0; j < ntiles && kb1 > kb0; ++j) {
      const int nbox = tile_nbox(j);
      const bool active = b < nbox;
      // FP32 partial sums for 8 features x NTOK tokens.  Each multiply-add is one
      // mixed-precision FMA on the 16-bit weight and activation (no conversion
      // instructions; same rounding as fmaf on the converted values).
      float acc[NTOK][8];
#pragma unroll
      for (int t = 0; t < NTOK; ++t)
#pragma unroll
        for (int jj = 0; jj < 8; ++jj) acc[t][jj] = 0.f;

      for (int kb = kb0; kb < kb1; ++kb, ++item) {
        const int s = item % S;
        const uint32_t ph = (uint32_t)((item / S) & 1);
        const bool ok = mbar_wait<false>(full0 + 8 * s, ph, wc);
        if (ok && active) {
          const uint8_t *wst = smem + L.w_off + s * kCoreWStageBytes + b * kCoreBoxBytes;
          const uint16_t *xst = reinterpret_cast<const uint16_t *>(smem + L.x_off + s * L.x_stage_stride);
#pragma unroll
          for (int i = 0; i < kCoreRowHalf / 8; ++i) {
            const int row = row0 + ro + 8 * i;
            const uint4 wv = *reinterpret_cast<const uint4 *>(wst + row * 128 + chunk_off);
            const uint32_t w2[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
            for (int t = 0; t < NTOK; ++t) {
              const uint16_t xh = xst[t * kCoreBK + row];
#pragma unroll
              for (int jj = 0; jj < 4; ++jj) Elem<T>::fma_pair(acc[t][2 * jj], acc[t][2 * jj + 1], w2[jj], xh);
            }
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(empty0 + 8 * s);
      }

      // Warp-shuffle reduction over the 8 row groups (lane bits 2..4).
#pragma unroll
      for (int t = 0; t < NTOK; ++t)
#pragma unroll
        for (int jj = 0; jj < 8; ++jj) {
          float v = acc[t][jj];
          v += __shfl_xor_sync(0xffffffffu, v, 4);
          v += __shfl_xor_sync(0xffffffffu, v, 8);
          v += __shfl_xor_sync(0xffffffffu, v, 16);
          acc[t][jj] = v;
        }
      // Lane (q, ro) now owns token ro of its 8 features.
      float out[8];
#pragma unroll
      for (int jj = 0; jj < 8; ++jj) out[jj] = 0.f;
#pragma unroll
      for (int t = 0; t < NTOK; ++t)
        if (t == ro)
#pragma unroll
          for (int jj = 0; jj < 8; ++jj) out[jj] = acc[t][jj];

      const int fcol = b * kBoxCols + c * 8;  // feature within the tile
      // Row half 1 hands its sums to row half 0 through a buffer chosen by tile
      // parity; the barrier of tile j + 1 keeps tile j's buffer until it is read.
      float *cb = comb + (size_t)(j & 1) * L.comb_floats + ro * kCoreBN + fcol;
      if (kq == 1 && ro < NTOK) {
        *reinterpret_cast<float4 *>(cb) = make_float4(out[0], out[1], out[2], out[3]);
        *reinterpret_cast<float4 *>(cb + 4) = make_float4(out[4], out[5], out[6], out[7]);
      }
      named_sync(1, kCoreConsumerWarps * 32);
      if (kq == 0) {
        if (ro < NTOK) {
          const float4 h0 = *reinterpret_cast<const float4 *>(cb);
          const float4 h1 = *reinterpret_cast<const float4 *>(cb + 4);
          out[0] += h0.x; out[1] += h0.y; out[2] += h0.z; out[3] += h0.w;
          out[4] += h1.x; out[5] += h1.y; out[6] += h1.z; out[7] += h1.w;
        }

        bool write_out = true;
        if (ks > 1) {
          if (r > 0) {
            // Member: push the partial into the leader's slot r-1.
            if (nred > 0) mbar_wait<true>(red_free, (uint32_t)((nred - 1) & 1), wc);
            const uint32_t leader = my_rank - (uint32_t)r;
            if (ro < NTOK) {
              const uint32_t dst = mapa_shared(
                  smem_u32(red + (size_t)(r - 1) * L.red_slot_floats + ro * kCoreBN + fcol), leader);
              st_cluster_v4(dst, out[0], out[1], out[2], out[3]);
              st_cluster_v4(dst + 16, out[4], out[5], out[6], out[7]);
            }
            mbar_arrive_remote(mapa_shared(red_full, leader));
            sent_remote = true;
            write_out = false;
          } else {
            // Leader: add the members' partials once all of them have landed.
            mbar_wait<true>(red_full, (uint32_t)(nred & 1), wc);
            if (ro < NTOK) {
              for (int m = 0; m < ks - 1; ++m) {
                const float *src = red + (size_t)m * L.red_slot_floats + ro * kCoreBN + fcol;
                const float4 a0 = *reinterpret_cast<const float4 *>(src);
                const float4 a1 = *reinterpret_cast<const float4 *>(src + 4);
                out[0] += a0.x; out[1] += a0.y; out[2] += a0.z; out[3] += a0.w;
                out[4] += a1.x; out[5] += a1.y; out[6] += a1.z; out[7] += a1.w;
              }
            }
            __syncwarp();
            // Members wait for this before sending their next partial; after
            // the last tile there is none, and a member may already have left.
            if (lane == 0 && j + 1 < ntiles)
              for (int m = 1; m < ks; ++m) mbar_arrive_remote(mapa_shared(red_free, my_rank + m));
          }
          ++nred;
        }

        if (write_out && active && ro < p.ntok) {
          const int col = tile_box0(j) * kBoxCols + fcol;
          if (col < tier.cols) {
            T *yrow = reinterpret_cast<T *>(p.y) + (long long)ro * p.ldy + tier.col_offset + col;
            if (col + 8 <= tier.cols && (reinterpret_cast<uintptr_t>(yrow) & 15u) == 0) {
              uint4 v;
              v.x = Elem<T>::pack2(out[0], out[1]);
              v.y = Elem<T>::pack2(out[2], out[3]);
              v.z = Elem<T>::pack2(out[4], out[5]);
              v.w = Elem<T>::pack2(out[6], out[7]);
              *reinterpret_cast<uint4 *>(yrow) = v;
            } else {
              uint16_t *yr = reinterpret_cast<uint16_t *>(yrow);
              for (int jj = 0; jj < 8 && col + jj < tier.cols; ++jj) yr[jj] = Elem<T>::from_float(out[jj]);
            }
          }
        }
      }
    }
  }
  // No CTA leaves while a peer may still touch its shared memory.  Members'
  // last partials were waited for by their leaders, and leaders send no
  // release after the last tile, so only the members' own remote writes need
  // release semantics; the output stores need none.
  cluster_exit_sync(sent_remote);
}

template <typename T>
cudaError_t launch_dtype(const LinearParams &p, int ntok_tmpl, int grid, int cluster, size_t smem,
                         cudaStream_t stream, int *mc) {
  switch (ntok_tmpl) {
    case 1: return launch_linear_kernel(linear_core_kernel<T, 1>, p, grid, kCoreThreads, cluster, smem, stream, mc);
    case 2: return launch_linear_kernel(linear_core_kernel<T, 2>, p, grid, kCoreThreads, cluster, smem, stream, mc);
    case 4: return launch_linear_kernel(linear_core_kernel<T, 4>, p, grid, kCoreThreads, cluster, smem, stream, mc);
    case 8: return launch_linear_kernel(linear_core_kernel<T, 8>, p, grid, kCoreThreads, cluster, smem, stream, mc);
    default: return cudaErrorInvalidValue;
  }
}

template <int NTOK>
size_t smem_for(int red_slots) {
  return CoreLayout<NTOK>(CoreLayout<NTOK>::stages_for(red_slots)).bytes(red_slots);
}

}  // namespace

int linear_core_stages(int ntok_tmpl, int red_slots) {
  switch (ntok_tmpl) {
    case 1: return CoreLayout<1>::stages_for(red_slots);
    case 2: return CoreLayout<2>::stages_for(red_slots);
    case 4: return CoreLayout<4>::stages_for(red_slots);
    case 8: return CoreLayout<8>::stages_for(red_slots);
    default: return 0;
  }
}

size_t linear_core_smem_bytes(int ntok_tmpl, int red_slots) {
  switch (ntok_tmpl) {
    case 1: return smem_for<1>(red_slots);
    case 2: return smem_for<2>(red_slots);
    case 4: return smem_for<4>(red_slots);
    case 8: return smem_for<8>(red_slots);
    default: return 0;
  }
}

cudaError_t launch_linear_core(const LinearParams &p, int ntok_tmpl, int dtype, int grid,
                               int cluster, size_t smem, cudaStream_t stream, int *max_clusters) {
  if (dtype == DAK_DTYPE_F16) return launch_dtype<__half>(p, ntok_tmpl, grid, cluster, smem, stream, max_clusters);
  if (dtype == DAK_DTYPE_BF16)
    return launch_dtype<__nv_bfloat16>(p, ntok_tmpl, grid, cluster, smem, stream, max_clusters);
  return cudaErrorInvalidValue;
}

}  // namespace dak
