// dak_attention.cu - split-KV decode attention over KV that lives partly in
// pinned host memory and partly in HBM, merged with log-sum-exp.
//
// Replaces opt_attention_decode_kernel / opt_attention_reduce_splits_kernel
// (opt_attention/csrc/opt_attention_kernel.cuh:260-386) and their launcher
// (opt_attention_kernel.cu:9-35).  The reference runs one CTA per
// (batch, query head, split) and so re-reads every K/V byte once per query
// head; it supports MHA, head_dim 128 and a per-batch-row host/device choice.
// Here:
//   * one CTA per (batch, KV head, split) serves all G = Hq/Hkv query heads of
//     the GQA group, so every KV byte crosses the host link or HBM once;
//   * K/V arrive as 64-token chunks through a 3-stage ring (two CTAs per SM,
//     so one CTA's start-up overlaps the other's stream) filled by TMA 4-D
//     tile loads (128-byte swizzle) issued by one producer warp; each chunk is
//     made of pages (64 tokens of one row in the reference's [B, H, S, D]
//     layout, or page_size-token pages of a paged pool), and each page picks
//     the host or the device tile map, so one sequence may span both tiers;
//   * 4 compute warps do q.k and p.V on the tensor cores (mma.sync m16n8k16,
//     FP32 accumulators; the group's query heads are the M rows) with an
//     online softmax (expf) per warp, merged across warps at the end;
//   * per-split (o, m, l) go to caller-provided FP32 scratch and a second
//     kernel merges the splits with log-sum-exp, as kernel.cuh:362-386 does.
#include <cfloat>

#include "dak_common.cuh"
#include "dak_host.h"

namespace dak {

namespace {

constexpr int kHeadDim = 128;
constexpr int kChunk = 64;          // tokens per pipeline stage
constexpr int kAttnStages = 3;      // ring depth: two CTAs share an SM
constexpr int kAttnComputeWarps = 4;
constexpr int kAttnThreads = (kAttnComputeWarps + 1) * 32;
constexpr int kMaxGroup = 8;
constexpr int kTabWindow = 256;     // block-table entries the producer caches in shared memory
constexpr uint32_t kHalfBox = kChunk * 128;              // 64 tokens x 64 dims x 2 B = 8 KB
constexpr uint32_t kKvChunkBytes = 2 * kHalfBox;        // 16 KB for K (or V)
constexpr uint32_t kStageBytes = 2 * kKvChunkBytes;     // K + V = 32 KB

struct alignas(64) AttnParams {
  CUtensorMap kmap[2];  // [0] host tier, [1] device tier; dims {128, rows, Hkv, n}
  CUtensorMap vmap[2];
  const void *query;
  long long q_stride_b, q_stride_h;
  const float *mask;
  long long mask_stride_b;
  void *out;
  long long o_stride_b, o_stride_h;
  float *partial_o;
  float *partial_ml;
  const int *block_table;  // paged mode; nullptr in batch-split mode
  long long bt_stride;
  const int *seq_lens;     // paged mode
  int batch, host_size, num_q_heads, num_kv_heads, seq_len, split_size, num_splits, page_size;
  float scaling;
  int *status;
  int pdl;                 // launched with programmatic stream serialization
  int *merge_counters;     // [batch * num_kv_heads]: the last split merges (nullptr: merge kernel)
  int check_pages;         // paged mode: bound table entries by pages[]
  long long pages[2];      // paged mode: pages in the [0] host, [1] device pool (0: no pool)
};

// Shared memory of a CTA with an ST-stage ring.  The warps' partial outputs
// (ored, 4 x G x 128 FP32), merged after the last chunk has been consumed,
// reuse the ring, so a 3-stage CTA needs about 98 KB and two CTAs share an
// SM: one CTA's start-up (barrier set-up, first TMA round trip) overlaps the
// other's stream.
template <int ST>
struct AttnSmem {
  static constexpr uint32_t kv_off = 0;
  static constexpr uint32_t ored_off = kv_off;                                           // 4 x G x 128
  static constexpr uint32_t redmax_off = kv_off + ST * kStageBytes;                      // 4 x G
  static constexpr uint32_t lred_off = redmax_off + kAttnComputeWarps * kMaxGroup * 4;  // 4 x G
  static constexpr uint32_t tab_off = lred_off + kAttnComputeWarps * kMaxGroup * 4;     // block-table window
  static constexpr uint32_t bar_off = tab_off + kTabWindow * 4;
  static constexpr uint32_t flag_off = bar_off + 2 * ST * 8;
  static constexpr uint32_t bytes = flag_off + 16 + 1024;
  static_assert(kAttnComputeWarps * kMaxGroup * kHeadDim * 4 <= ST * kStageBytes, "ored must fit in the ring");
};
// Two CTAs (plus the 1 KB the SM reserves for each) share an SM's 228 KB.
static_assert(2 * (AttnSmem<kAttnStages>::bytes + 1024) <= 228 * 1024, "the ring must let two CTAs share an SM");

__device__ __forceinline__ void tma_load_4d(uint32_t dst, const CUtensorMap *map, int c0, int c1, int c2,
                                            int c3, uint32_t bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      ".L2::cache_hint [%0], [%1, {%2, %3, %4, %5}], [%6], %7;" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(bar), "l"(policy)
      : "memory");
}

// Four 8x8 16-bit matrices from shared memory (row addresses from lanes 8j..8j+7
// for matrix j), optionally transposed; the operand loads of mma.sync.
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}

// D = A (16x16, row) * B (16x8, col) + D with 16-bit inputs and FP32 accumulators.
template <typename T> struct Mma;
template <> struct Mma<__half> {
  static __device__ __forceinline__ void run(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
                 "{%8, %9}, {%0, %1, %2, %3};"
                 : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
                 : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
};
template <> struct Mma<__nv_bfloat16> {
  static __device__ __forceinline__ void run(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
                 "{%8, %9}, {%0, %1, %2, %3};"
                 : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
                 : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
};

// Where page j (page_size tokens) of sequence b lives: tier (0 host, 1 device),
// the row offset inside the tile map's second dimension and the slab index
// (4th dimension).
struct PageLoc {
  int tier, row, slab;
};

__device__ __forceinline__ PageLoc locate(const AttnParams &p, int b, int tok0) {
  PageLoc l;
  if (p.block_table) {
    const int v = p.block_table[(long long)b * p.bt_stride + tok0 / p.page_size];
    l.tier = v < 0 ? 0 : 1;
    l.slab = v < 0 ? (-1 - v) : v;
    l.row = 0;
  } else {
    l.tier = b < p.host_size ? 0 : 1;
    l.slab = b < p.host_size ? b : b - p.host_size;
    l.row = tok0;
  }
  return l;
}

// Log-sum-exp merge of the split partials (opt_attention_kernel.cuh:362-386).
// Both merge paths below compute, for each head, in split order and with the
// same fused multiply-adds:
//   gm = max_s m_s,  c_s = exp(m_s - gm) (0 for an empty split),
//   den = sum_s l_s c_s,  out_d = (sum_s o_{s,d} c_s) / den (0 when den == 0),
// so the separate merge kernel and the in-kernel merge give the same bits.
// The partials are read through L2: other CTAs wrote them.
__device__ __forceinline__ float merge_scale(float m, float gm) {
  return (m == -FLT_MAX || gm == -FLT_MAX) ? 0.f : expf(m - gm);
}

// One query head per CTA, dim d per thread (the merge kernel).
template <typename T>
__device__ __forceinline__ void merge_one_head(const AttnParams &p, int b, int hq, int d) {
  const long long base = ((long long)b * p.num_q_heads + hq) * p.num_splits;
  float gm = -FLT_MAX;
  for (int s = 0; s < p.num_splits; ++s) gm = fmaxf(gm, __ldcg(p.partial_ml + (base + s) * 2));
  float den = 0.f, acc = 0.f;
  for (int s = 0; s < p.num_splits; ++s) {
    const float c = merge_scale(__ldcg(p.partial_ml + (base + s) * 2), gm);
    den = __fmaf_rn(__ldcg(p.partial_ml + (base + s) * 2 + 1), c, den);
    acc = __fmaf_rn(__ldcg(p.partial_o + (base + s) * kHeadDim + d), c, acc);
  }
  uint16_t *out = reinterpret_cast<uint16_t *>(p.out) + (long long)b * p.o_stride_b + (long long)hq * p.o_stride_h;
  out[d] = Elem<T>::from_float(den == 0.f ? 0.f : acc / den);
}

// Shared-memory floats the in-kernel merge of G heads over `splits` needs:
// (m, l) pairs, scales and one denominator per head.
__host__ __device__ constexpr long long merge_stage_floats(int G, long long splits) {
  return 3 * G * splits + G;
}

// The G query heads of KV head kvh of sequence b, by the 128 compute threads
// of the CTA that finished last, with `stage` (shared memory) for the (m, l)
// pairs and scales.  The pairs arrive in one parallel load, one thread per
// head turns them into scales, and each thread then sums its dim of all G
// heads with G independent loads per split, so the merge costs a few L2 round
// trips rather than one per split and head.
template <typename T, int G>
__device__ __forceinline__ void merge_group(const AttnParams &p, int b, int kvh, float *stage) {
  const int S = p.num_splits;
  const int tid = threadIdx.x;
  float *ml = stage;             // [G][S][2]
  float *sc = stage + 2 * G * S; // [G][S]
  float *den = sc + G * S;       // [G]
  // Heads kvh*G .. kvh*G+G-1 of sequence b are contiguous in the partials.
  const long long base = ((long long)b * p.num_q_heads + (long long)kvh * G) * S;
  for (int i = tid; i < 2 * G * S; i += kAttnComputeWarps * 32) ml[i] = __ldcg(p.partial_ml + base * 2 + i);
  named_sync(1, kAttnComputeWarps * 32);
  if (tid < G) {
    const float *mg = ml + (long long)tid * S * 2;
    float gm = -FLT_MAX;
    for (int s = 0; s < S; ++s) gm = fmaxf(gm, mg[2 * s]);
    float dn = 0.f;
    for (int s = 0; s < S; ++s) {
      const float c = merge_scale(mg[2 * s], gm);
      sc[tid * S + s] = c;
      dn = __fmaf_rn(mg[2 * s + 1], c, dn);
    }
    den[tid] = dn;
  }
  named_sync(1, kAttnComputeWarps * 32);
  const int d = tid;
  const float *po = p.partial_o + base * kHeadDim + d;
  float acc[G];
#pragma unroll
  for (int g = 0; g < G; ++g) acc[g] = 0.f;
#pragma unroll 2
  for (int s = 0; s < S; ++s) {
#pragma unroll
    for (int g = 0; g < G; ++g)
      acc[g] = __fmaf_rn(__ldcg(po + ((long long)g * S + s) * kHeadDim), sc[g * S + s], acc[g]);
  }
  uint16_t *out = reinterpret_cast<uint16_t *>(p.out) + (long long)b * p.o_stride_b;
#pragma unroll
  for (int g = 0; g < G; ++g)
    out[(long long)(kvh * G + g) * p.o_stride_h + d] = Elem<T>::from_float(den[g] == 0.f ? 0.f : acc[g] / den[g]);
}

template <typename T, int G, int ST>
__global__ void __launch_bounds__(kAttnThreads, 1) attn_decode_kernel(const __grid_constant__ AttnParams p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_u32 = smem_u32(smem_raw);
  uint8_t *smem = smem_raw + (((raw_u32 + 1023u) & ~1023u) - raw_u32);
  const uint32_t sbase = smem_u32(smem);
  using S = AttnSmem<ST>;
  pdl_enter(p.pdl);  // q, the newest K/V and seq_lens come from the kernels before

  const int warp = warp_id();
  const int lane = lane_id();
  const int split = blockIdx.x % p.num_splits;
  const int kvh = (blockIdx.x / p.num_splits) % p.num_kv_heads;
  const int b = blockIdx.x / (p.num_splits * p.num_kv_heads);
  const int seq = p.seq_lens ? min(p.seq_lens[b], p.seq_len) : p.seq_len;
  const int t_begin = split * p.split_size;
  const int t_end = min(seq, t_begin + p.split_size);
  const int nchunks = t_end > t_begin ? (t_end - t_begin + kChunk - 1) / kChunk : 0;

  float *redmax = reinterpret_cast<float *>(smem + S::redmax_off);
  float *ored = reinterpret_cast<float *>(smem + S::ored_off);
  float *lred = reinterpret_cast<float *>(smem + S::lred_off);
  const uint32_t full0 = sbase + S::bar_off;
  const uint32_t empty0 = full0 + ST * 8;
  volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + S::flag_off);
  const WaitCtx wc{abort_flag, p.status};

  if (threadIdx.x == 0) {
    for (int s = 0; s < ST; ++s) {
      mbar_init(full0 + 8 * s, 1);
      mbar_init(empty0 + 8 * s, kAttnComputeWarps);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == kAttnComputeWarps) {
    // ------------------------------------------------------------ producer
    // Lane 0 issues the copies.  In paged mode the whole warp first loads a
    // window of the split's block-table entries into shared memory with one
    // coalesced pass, so no copy waits on a dependent global load.
    if (nchunks > 0) {
      if (lane == 0)
        for (int t = 0; t < 2; ++t) {
          prefetch_tensormap(&p.kmap[t]);
          prefetch_tensormap(&p.vmap[t]);
        }
      const uint64_t pol = l2_policy_evict_first();
      const int psz = p.block_table ? p.page_size : kChunk;
      int *tab_s = reinterpret_cast<int *>(smem + S::tab_off);
      const int seq_pages = (t_end + psz - 1) / psz;  // table entries this split may read
      int win = -kTabWindow;                          // first page held in tab_s
      uint32_t issued_mask = 0, issued_par = 0;
      for (int c = 0; c < nchunks; ++c) {
        const int s = c % ST;
        const uint32_t ph = (uint32_t)((c / ST) & 1);
        const int c0 = t_begin + c * kChunk;
        const int valid = min(kChunk, t_end - c0);
        const int npages = (valid + psz - 1) / psz;
        const int pfirst = c0 / psz;
        if (p.block_table && pfirst + npages > win + kTabWindow) {
          win = pfirst;
          __syncwarp();
          for (int i = lane; i < kTabWindow && win + i < seq_pages; i += 32)
            tab_s[i] = p.block_table[(long long)b * p.bt_stride + win + i];
          __syncwarp();
        }
        int ok = 1;
        if (lane == 0) {
          ok = mbar_wait<false>(empty0 + 8 * s, ph ^ 1u, wc) ? 1 : 0;
          if (ok) {
            const uint32_t fb = full0 + 8 * s;
            mbar_arrive_expect_tx(fb, (uint32_t)npages * (uint32_t)psz * 128u * 4u);
            const uint32_t kdst = sbase + S::kv_off + s * kStageBytes;
            const uint32_t vdst = kdst + kKvChunkBytes;
            for (int pg = 0; pg < npages; ++pg) {
              PageLoc loc;
              if (p.block_table) {
                const int v = tab_s[pfirst + pg - win];
                loc.tier = v < 0 ? 0 : 1;
                loc.slab = v < 0 ? (-1 - v) : v;
                loc.row = 0;
                if (p.check_pages && loc.slab >= p.pages[loc.tier]) {
                  // Past the pool (or no pool): one past the tile map's last
                  // page, so the copy reads zeros and still completes.
                  atomicCAS(p.status, 0, DAK_ERR_INVALID_ARG);
                  loc.slab = (int)max(1ll, p.pages[loc.tier]);
                }
              } else {
                loc = locate(p, b, c0 + pg * psz);
              }
              const uint32_t row_off = (uint32_t)(pg * psz) * 128u;
              for (int h = 0; h < 2; ++h) {
                tma_load_4d(kdst + h * kHalfBox + row_off, &p.kmap[loc.tier], h * 64, loc.row, kvh, loc.slab, fb, pol);
                tma_load_4d(vdst + h * kHalfBox + row_off, &p.vmap[loc.tier], h * 64, loc.row, kvh, loc.slab, fb, pol);
              }
            }
            issued_mask |= 1u << s;
            issued_par = (issued_par & ~(1u << s)) | (ph << s);
          }
        }
        if (!__shfl_sync(0xffffffffu, ok, 0)) break;
      }
      if (lane == 0 && *abort_flag) {
        const WaitCtx drain{reinterpret_cast<volatile int *>(smem + S::flag_off + 4), p.status};
        *drain.abort = 0;
        for (int st = 0; st < ST; ++st)
          if (issued_mask & (1u << st)) mbar_wait<false>(full0 + 8 * st, (issued_par >> st) & 1u, drain);
      }
    }
    __syncwarp();
    return;
  }

  // ---------------------------------------------------------------- compute
  // Tensor cores (mma.sync m16n8k16, FP32 accumulators).  Warp w owns tokens
  // 16w .. 16w+15 of every chunk and keeps its own online softmax; the four
  // warps' (m, l, o) are merged once at the end.  The G query heads of the
  // group are the M rows (rows G..15 are zero):
  //   S[16 x 16 tokens] = Q[16 x 128] . K^T      (8 k-steps x 2 token tiles)
  //   O[16 x 128]      += P[16 x 16] . V[16 x 128] (16 dim tiles)
  // P is rounded to the input type before P.V, as transformers' eager path
  // does (softmax in FP32, then cast to the query dtype).
  const int r = lane >> 2;   // fragment row: query head
  const int cq = lane & 3;   // fragment column pair
  const int tw = 16 * warp;  // this warp's first token in a chunk
  uint32_t qa[8][4];
  {
    const uint32_t *qrow = nullptr;
    if (r < G)
      qrow = reinterpret_cast<const uint32_t *>(reinterpret_cast<const uint16_t *>(p.query) + (long long)b * p.q_stride_b +
                                                (long long)(kvh * G + r) * p.q_stride_h);
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
      qa[ks][0] = qrow ? qrow[(ks * 16 + cq * 2) / 2] : 0u;
      qa[ks][1] = 0u;  // rows 8..15
      qa[ks][2] = qrow ? qrow[(ks * 16 + cq * 2 + 8) / 2] : 0u;
      qa[ks][3] = 0u;
    }
  }
  float m_run = -FLT_MAX, l_part = 0.f;  // row r of this warp
  float o[16][4];
#pragma unroll
  for (int nt = 0; nt < 16; ++nt)
#pragma unroll
    for (int j = 0; j < 4; ++j) o[nt][j] = 0.f;

  for (int c = 0; c < nchunks; ++c) {
    const int s = c % ST;
    const uint32_t ph = (uint32_t)((c / ST) & 1);
    const bool ok = mbar_wait<false>(full0 + 8 * s, ph, wc);
    const uint32_t kst = sbase + S::kv_off + s * kStageBytes;
    const uint32_t vst = kst + kKvChunkBytes;
    const int c0 = t_begin + c * kChunk;
    const int valid = ok ? min(kChunk, t_end - c0) : 0;
    if (valid < kChunk) {
      // Rows past the end hold stale bytes that P = 0 would still multiply:
      // clear them (both 64-dim halves of V) before any warp reads V.
      uint8_t *vgen = smem + S::kv_off + s * kStageBytes + kKvChunkBytes;
      for (int i = threadIdx.x; i < (kChunk - valid) * 16; i += kAttnComputeWarps * 32) {
        const int row = valid + i / 16, piece = i % 16;
        *reinterpret_cast<uint4 *>(vgen + (piece >> 3) * kHalfBox + row * 128 + (piece & 7) * 16) =
            make_uint4(0u, 0u, 0u, 0u);
      }
      named_sync(1, kAttnComputeWarps * 32);
    }

    if (tw < valid) {
      // ---- S = Q . K^T for tokens tw .. tw+15
      float sc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        // matrix j: tokens tw + 8*(j>>1) + (lane&7), 8 dims at 16-byte chunk (ks%4)*2 + (j&1)
        const int j = lane >> 3;
        const int row = tw + 8 * (j >> 1) + (lane & 7);
        const int ch = (ks & 3) * 2 + (j & 1);
        const uint32_t addr = kst + (ks >> 2) * kHalfBox + row * 128 + ((ch ^ (row & 7)) << 4);
        uint32_t b00, b01, b10, b11;
        ldsm_x4(addr, b00, b01, b10, b11);
        Mma<T>::run(sc[0], qa[ks], b00, b01);
        Mma<T>::run(sc[1], qa[ks], b10, b11);
      }
      // ---- online softmax of row r over this warp's 16 tokens
      float v[4];
      float mx = -FLT_MAX;
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int t = tw + nt * 8 + cq * 2 + e;
          float x = sc[nt][e] * p.scaling;
          if (p.mask && t < valid) x += p.mask[(long long)b * p.mask_stride_b + c0 + t];
          x = t < valid ? x : -FLT_MAX;
          v[nt * 2 + e] = x;
          mx = fmaxf(mx, x);
        }
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      const float mn = fmaxf(m_run, mx);
      const float alpha = (m_run == -FLT_MAX) ? 0.f : expf(m_run - mn);
      float pr[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) pr[e] = (v[e] == -FLT_MAX || mn == -FLT_MAX) ? 0.f : expf(v[e] - mn);
      m_run = mn;
      // Round P to the input type; l sums the rounded values P.V will use.
      uint32_t pa[4];
      pa[0] = Elem<T>::pack2(pr[0], pr[1]);
      pa[1] = 0u;
      pa[2] = Elem<T>::pack2(pr[2], pr[3]);
      pa[3] = 0u;
      {
        const float2 p01 = Elem<T>::to_float2(pa[0]), p23 = Elem<T>::to_float2(pa[2]);
        l_part = l_part * alpha + (p01.x + p01.y + p23.x + p23.y);
      }
#pragma unroll
      for (int nt = 0; nt < 16; ++nt) {
        o[nt][0] *= alpha;
        o[nt][1] *= alpha;
      }
      // ---- O += P . V over tokens tw .. tw+15, dims in 16 tiles of 8
#pragma unroll
      for (int np = 0; np < 8; ++np) {
        // matrix j: tokens tw + 8*(j&1) + (lane&7), dims chunk 2*np + (j>>1) (transposed)
        const int j = lane >> 3;
        const int row = tw + 8 * (j & 1) + (lane & 7);
        const int dch = 2 * np + (j >> 1);
        const uint32_t addr = vst + (dch >> 3) * kHalfBox + row * 128 + (((dch & 7) ^ (row & 7)) << 4);
        uint32_t b0a, b1a, b0b, b1b;
        ldsm_x4_t(addr, b0a, b1a, b0b, b1b);
        Mma<T>::run(o[2 * np], pa, b0a, b1a);
        Mma<T>::run(o[2 * np + 1], pa, b0b, b1b);
      }
    }
    if (valid < kChunk) {
      // The stage's next fill comes from the async proxy.
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(empty0 + 8 * s);
  }

  // ---- merge the 4 warps: row r of warp w holds (m, l, o[dims])
  float l = l_part;
  l += __shfl_xor_sync(0xffffffffu, l, 1);
  l += __shfl_xor_sync(0xffffffffu, l, 2);
  float *mred = redmax;                                  // [warp][G]
  float *lr = lred;                                      // [warp][G]
  // ored reuses the ring: every warp must be done reading its last chunk.
  named_sync(1, kAttnComputeWarps * 32);
  if (r < G) {
    if (cq == 0) {
      mred[warp * kMaxGroup + r] = m_run;
      lr[warp * kMaxGroup + r] = l;
    }
#pragma unroll
    for (int nt = 0; nt < 16; ++nt)
      *reinterpret_cast<float2 *>(ored + (warp * kMaxGroup + r) * kHeadDim + nt * 8 + cq * 2) =
          make_float2(o[nt][0], o[nt][1]);
  }
  named_sync(1, kAttnComputeWarps * 32);
  // Thread tid finishes dim tid of every head.
  const int d = threadIdx.x;
  for (int g = 0; g < G; ++g) {
    float gm = -FLT_MAX;
#pragma unroll
    for (int w = 0; w < kAttnComputeWarps; ++w) gm = fmaxf(gm, mred[w * kMaxGroup + g]);
    float acc = 0.f, den = 0.f;
#pragma unroll
    for (int w = 0; w < kAttnComputeWarps; ++w) {
      const float mw = mred[w * kMaxGroup + g];
      const float sc = (mw == -FLT_MAX) ? 0.f : expf(mw - gm);
      acc += ored[(w * kMaxGroup + g) * kHeadDim + d] * sc;
      den += lr[w * kMaxGroup + g] * sc;
    }
    const int hq = kvh * G + g;
    if (p.num_splits == 1) {
      uint16_t *out = reinterpret_cast<uint16_t *>(p.out) + (long long)b * p.o_stride_b + (long long)hq * p.o_stride_h;
      out[d] = Elem<T>::from_float(den == 0.f ? 0.f : acc / den);
    } else {
      const long long base = ((long long)b * p.num_q_heads + hq) * p.num_splits + split;
      p.partial_o[base * kHeadDim + d] = acc;
      if (d == 0) {
        p.partial_ml[base * 2] = gm;
        p.partial_ml[base * 2 + 1] = den;
      }
    }
  }
  if (p.num_splits > 1 && p.merge_counters) {
    // The last split of this (sequence, KV head) to finish merges all of them:
    // every CTA publishes its partials, then counts itself; the CTA that
    // counts last sees every partial and resets the counter for the next call.
    int *last = reinterpret_cast<int *>(smem + S::flag_off + 8);
    __threadfence();
    named_sync(1, kAttnComputeWarps * 32);
    if (threadIdx.x == 0) {
      int *counter = p.merge_counters + (long long)b * p.num_kv_heads + kvh;
      *last = atomicAdd(counter, 1) == p.num_splits - 1 ? 1 : 0;
      if (*last) *counter = 0;
    }
    named_sync(1, kAttnComputeWarps * 32);
    if (*last) {
      __threadfence();
      // The ring is free: every thread is past its last read of ored.
      merge_group<T, G>(p, b, kvh, reinterpret_cast<float *>(smem + S::kv_off));
    }
  }
}

// Log-sum-exp merge of the splits (opt_attention_kernel.cuh:362-386).
template <typename T>
__global__ void __launch_bounds__(kHeadDim) attn_merge_kernel(const __grid_constant__ AttnParams p) {
  pdl_enter(p.pdl);
  merge_one_head<T>(p, blockIdx.x / p.num_q_heads, blockIdx.x % p.num_q_heads, threadIdx.x);
}

template <typename T, int G, int ST>
cudaError_t launch_g(const AttnParams &p, cudaStream_t stream) {
  auto kern = attn_decode_kernel<T, G, ST>;
  constexpr uint32_t smem = AttnSmem<ST>::bytes;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  const int grid = p.batch * p.num_kv_heads * p.num_splits;
  e = launch_ex(kern, dim3(grid), dim3(kAttnThreads), smem, stream, 1, p.pdl != 0, p);
  if (e != cudaSuccess || p.num_splits == 1 || p.merge_counters) return e;
  return launch_ex(attn_merge_kernel<T>, dim3(p.batch * p.num_q_heads), dim3(kHeadDim), 0, stream, 1, p.pdl != 0, p);
}

template <typename T>
cudaError_t launch_t(const AttnParams &p, int group, cudaStream_t stream) {
  switch (group) {
    case 1: return launch_g<T, 1, kAttnStages>(p, stream);
    case 2: return launch_g<T, 2, kAttnStages>(p, stream);
    case 4: return launch_g<T, 4, kAttnStages>(p, stream);
    case 8: return launch_g<T, 8, kAttnStages>(p, stream);
    default: return cudaErrorInvalidValue;
  }
}

// 4-D tile map over K or V: dims {128, rows, Hkv, slabs}; box {64, box_rows, 1, 1}.
int kv_map(CUtensorMap *out, const void *base, int dtype, long long rows, long long heads, long long slabs,
           long long stride_row, long long stride_head, long long stride_slab, int box_rows);

}  // namespace

}  // namespace dak

// ------------------------------------------------------------------ C ABI
#include <cudaTypedefs.h>

#include <cstring>
#include <mutex>

namespace dak {
namespace {

PFN_cuTensorMapEncodeTiled_v12000 attn_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, []() {
    void *ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &ptr, 12000, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}

int kv_map(CUtensorMap *out, const void *base, int dtype, long long rows, long long heads, long long slabs,
           long long stride_row, long long stride_head, long long stride_slab, int box_rows) {
  int st = check_gpu_accessible(base, "KV");
  if (st) return st;
  auto fn = attn_encode_fn();
  if (!fn) return fail(DAK_ERR_DRIVER, "cuTensorMapEncodeTiled entry point unavailable");
  const cuuint64_t gdim[4] = {(cuuint64_t)kHeadDim, (cuuint64_t)rows, (cuuint64_t)heads, (cuuint64_t)slabs};
  const cuuint64_t gstride[3] = {(cuuint64_t)stride_row * 2u, (cuuint64_t)stride_head * 2u,
                                 (cuuint64_t)stride_slab * 2u};
  const cuuint32_t box[4] = {64u, (cuuint32_t)box_rows, 1u, 1u};
  const cuuint32_t es[4] = {1, 1, 1, 1};
  CUresult r = fn(out, dtype == DAK_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                  4, const_cast<void *>(base), gdim, gstride, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(DAK_ERR_DRIVER, "cuTensorMapEncodeTiled (KV) failed with %d", (int)r);
  return DAK_OK;
}

int check_kv_strides(const void *ptr, long long sb, long long sh, const char *what) {
  if (!ptr) return fail(DAK_ERR_INVALID_ARG, "%s is null", what);
  if ((reinterpret_cast<uintptr_t>(ptr) & 15u) != 0) return fail(DAK_ERR_ALIGNMENT, "%s must be 16-byte aligned", what);
  if (sb <= 0 || sh <= 0 || (sb % 8) != 0 || (sh % 8) != 0)
    return fail(DAK_ERR_ALIGNMENT, "%s batch/head strides must be positive multiples of 8 elements", what);
  return DAK_OK;
}

int common_checks(int batch, int hq, int hkv, int head_dim, int split_size, int dtype, int *group) {
  if (dtype != DAK_DTYPE_F16 && dtype != DAK_DTYPE_BF16)
    return fail(DAK_ERR_UNSUPPORTED, "attention supports float16 and bfloat16 only");
  if (head_dim != kHeadDim) return fail(DAK_ERR_UNSUPPORTED, "decode kernel requires head_dim == 128");
  if (batch <= 0 || hq <= 0 || hkv <= 0) return fail(DAK_ERR_INVALID_ARG, "batch and head counts must be positive");
  if (hq % hkv != 0) return fail(DAK_ERR_INVALID_ARG, "num_q_heads must be a multiple of num_kv_heads");
  const int g = hq / hkv;
  if (g != 1 && g != 2 && g != 4 && g != 8)
    return fail(DAK_ERR_UNSUPPORTED, "query heads per KV head must be 1, 2, 4 or 8 (got %d)", g);
  if (split_size <= 0 || split_size % kChunk != 0)
    return fail(DAK_ERR_INVALID_ARG, "split_size must be a positive multiple of 64");
  *group = g;
  return DAK_OK;
}

}  // namespace
}  // namespace dak

using namespace dak;

extern "C" {

int dak_attn_decode(const dak_attn_decode_args *a, void *stream) {
  if (!a) return fail(DAK_ERR_INVALID_ARG, "args is null");
  int group, st;
  if ((st = common_checks(a->batch, a->num_q_heads, a->num_kv_heads, a->head_dim, a->split_size, a->dtype, &group)))
    return st;
  if (a->host_size < 0 || a->host_size > a->batch)
    return fail(DAK_ERR_INVALID_ARG, "host_size must be in [0, batch_size], got %d for batch_size=%d", a->host_size,
                a->batch);
  if (a->seq_len <= 0) return fail(DAK_ERR_INVALID_ARG, "seq_len must be positive");
  if (!a->query || !a->out) return fail(DAK_ERR_INVALID_ARG, "query and out are required");
  const int gpu_batch = a->batch - a->host_size;
  AttnParams p;
  std::memset(&p, 0, sizeof(p));
  p.pdl = decode_pdl_enabled() ? 1 : 0;
  if (gpu_batch > 0) {
    if ((st = check_kv_strides(a->key, a->kv_stride_b, a->kv_stride_h, "key"))) return st;
    if ((st = check_kv_strides(a->value, a->kv_stride_b, a->kv_stride_h, "value"))) return st;
    if ((st = kv_map(&p.kmap[1], a->key, a->dtype, a->seq_len, a->num_kv_heads, gpu_batch, kHeadDim, a->kv_stride_h,
                     a->kv_stride_b, kChunk)))
      return st;
    if ((st = kv_map(&p.vmap[1], a->value, a->dtype, a->seq_len, a->num_kv_heads, gpu_batch, kHeadDim,
                     a->kv_stride_h, a->kv_stride_b, kChunk)))
      return st;
  }
  if (a->host_size > 0) {
    if ((st = check_kv_strides(a->key_host, a->kvh_stride_b, a->kvh_stride_h, "key_host"))) return st;
    if ((st = check_kv_strides(a->value_host, a->kvh_stride_b, a->kvh_stride_h, "value_host"))) return st;
    if ((st = kv_map(&p.kmap[0], a->key_host, a->dtype, a->seq_len, a->num_kv_heads, a->host_size, kHeadDim,
                     a->kvh_stride_h, a->kvh_stride_b, kChunk)))
      return st;
    if ((st = kv_map(&p.vmap[0], a->value_host, a->dtype, a->seq_len, a->num_kv_heads, a->host_size, kHeadDim,
                     a->kvh_stride_h, a->kvh_stride_b, kChunk)))
      return st;
  }
  const int splits = (a->seq_len + a->split_size - 1) / a->split_size;
  if (splits > 1 && (!a->partial_o || !a->partial_ml))
    return fail(DAK_ERR_INVALID_ARG, "partial_o and partial_ml scratch are required when seq_len > split_size");
  p.query = a->query;
  p.q_stride_b = a->q_stride_b;
  p.q_stride_h = a->q_stride_h;
  p.mask = a->mask;
  p.mask_stride_b = a->mask_stride_b;
  p.out = a->out;
  p.o_stride_b = a->o_stride_b;
  p.o_stride_h = a->o_stride_h;
  p.partial_o = a->partial_o;
  p.partial_ml = a->partial_ml;
  p.batch = a->batch;
  p.host_size = a->host_size;
  p.num_q_heads = a->num_q_heads;
  p.num_kv_heads = a->num_kv_heads;
  p.seq_len = a->seq_len;
  p.split_size = a->split_size;
  p.num_splits = splits;
  p.page_size = kChunk;
  p.scaling = a->scaling;
  p.status = device_status_word();
  if (!p.status) return fail(DAK_ERR_CUDA, "no device status word");
  cudaError_t e = a->dtype == DAK_DTYPE_F16 ? launch_t<__half>(p, group, static_cast<cudaStream_t>(stream))
                                            : launch_t<__nv_bfloat16>(p, group, static_cast<cudaStream_t>(stream));
  return cuda_status(e, "attention launch");
}

}  // extern "C"

namespace dak {
namespace {
// Both paged entry points: with merge_counters the last split of each
// (sequence, KV head) merges the partials inside the attention kernel.
int attn_paged(const dak_attn_paged_args *a, int32_t *merge_counters, void *stream) {
  if (!a) return fail(DAK_ERR_INVALID_ARG, "args is null");
  int group, st;
  if ((st = common_checks(a->batch, a->num_q_heads, a->num_kv_heads, a->head_dim, a->split_size, a->dtype, &group)))
    return st;
  if (a->page_size != 16 && a->page_size != 32 && a->page_size != 64)
    return fail(DAK_ERR_UNSUPPORTED, "page_size must be 16, 32 or 64");
  if (a->max_seq_len <= 0 || !a->block_table || !a->seq_lens || a->bt_stride <= 0)
    return fail(DAK_ERR_INVALID_ARG, "block_table, seq_lens and max_seq_len are required");
  if ((long long)a->bt_stride * a->page_size < a->max_seq_len)
    return fail(DAK_ERR_INVALID_ARG, "block_table rows are shorter than max_seq_len pages");
  if (!a->query || !a->out) return fail(DAK_ERR_INVALID_ARG, "query and out are required");
  AttnParams p;
  std::memset(&p, 0, sizeof(p));
  p.pdl = decode_pdl_enabled() ? 1 : 0;
  const long long hs = (long long)a->page_size * kHeadDim;      // head stride in a page
  const long long ps = hs * a->num_kv_heads;                     // page stride
  if (!a->k_pool_dev && !a->k_pool_host) return fail(DAK_ERR_INVALID_ARG, "no KV pool given");
  if (a->dev_pages < 0 || a->host_pages < 0) return fail(DAK_ERR_INVALID_ARG, "page counts must not be negative");
  // With page counts, each map covers exactly its pool and the kernel bounds
  // every table entry; a tier without a pool gets a one-page map over the
  // other tier's pool that no entry reaches.  Without them, the maps cover the
  // largest page index a 31-bit table entry can name and entries are trusted.
  p.check_pages = (a->dev_pages > 0 || a->host_pages > 0) ? 1 : 0;
  p.pages[0] = a->k_pool_host ? a->host_pages : 0;
  p.pages[1] = a->k_pool_dev ? a->dev_pages : 0;
  const long long max_pages = 1ll << 24;
  const void *pools[4] = {a->k_pool_host, a->v_pool_host, a->k_pool_dev, a->v_pool_dev};
  for (int i = 0; i < 4; ++i) {
    const int tier = i < 2 ? 0 : 1;
    const void *base = pools[i] ? pools[i] : (p.check_pages ? pools[i ^ 2] : nullptr);
    if (!base) continue;
    if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0) return fail(DAK_ERR_ALIGNMENT, "KV pools must be 16-byte aligned");
    const long long slabs = p.check_pages ? std::max(1ll, p.pages[tier]) : max_pages;
    CUtensorMap *m = (i % 2 == 0) ? &p.kmap[tier] : &p.vmap[tier];
    if ((st = kv_map(m, base, a->dtype, a->page_size, a->num_kv_heads, slabs, kHeadDim, hs, ps, a->page_size)))
      return st;
  }
  const int splits = (a->max_seq_len + a->split_size - 1) / a->split_size;
  if (splits > 1 && (!a->partial_o || !a->partial_ml))
    return fail(DAK_ERR_INVALID_ARG, "partial_o and partial_ml scratch are required when max_seq_len > split_size");
  p.query = a->query;
  p.q_stride_b = a->q_stride_b;
  p.q_stride_h = a->q_stride_h;
  p.out = a->out;
  p.o_stride_b = a->o_stride_b;
  p.o_stride_h = a->o_stride_h;
  p.partial_o = a->partial_o;
  p.partial_ml = a->partial_ml;
  p.block_table = a->block_table;
  p.bt_stride = a->bt_stride;
  p.seq_lens = a->seq_lens;
  p.batch = a->batch;
  p.host_size = 0;
  p.num_q_heads = a->num_q_heads;
  p.num_kv_heads = a->num_kv_heads;
  p.seq_len = a->max_seq_len;
  p.split_size = a->split_size;
  p.num_splits = splits;
  p.page_size = a->page_size;
  p.scaling = a->scaling;
  p.status = device_status_word();
  if (!p.status) return fail(DAK_ERR_CUDA, "no device status word");
  if (merge_counters && splits > 1) {
    if ((reinterpret_cast<uintptr_t>(merge_counters) & 3u) != 0)
      return fail(DAK_ERR_ALIGNMENT, "merge_counters must be 4-byte aligned");
    cudaPointerAttributes attr;
    if (cudaPointerGetAttributes(&attr, merge_counters) != cudaSuccess || attr.type != cudaMemoryTypeDevice) {
      cudaGetLastError();
      return fail(DAK_ERR_INVALID_ARG, "merge_counters must be device memory of the current device");
    }
    // A merge whose (m, l) pairs and scales do not fit the ring (more than
    // about 8K splits x heads per KV head) takes the separate merge kernel
    // and leaves the counters untouched.
    if (merge_stage_floats(group, splits) * 4 <= (long long)kAttnStages * kStageBytes) p.merge_counters = merge_counters;
  }
  cudaError_t e = a->dtype == DAK_DTYPE_F16 ? launch_t<__half>(p, group, static_cast<cudaStream_t>(stream))
                                            : launch_t<__nv_bfloat16>(p, group, static_cast<cudaStream_t>(stream));
  return cuda_status(e, "paged attention launch");
}
}  // namespace
}  // namespace dak

extern "C" {

int dak_attn_decode_paged(const dak_attn_paged_args *a, void *stream) {
  return dak::attn_paged(a, nullptr, stream);
}

int dak_attn_decode_paged_merged(const dak_attn_paged_args *a, int32_t *merge_counters, void *stream) {
  if (!merge_counters) return dak::fail(DAK_ERR_INVALID_ARG, "merge_counters is null");
  return dak::attn_paged(a, merge_counters, stream);
}

}  // extern "C"

// ------------------------------------------------- allocation-free variant
// dak_attn_decode needs the caller to pass FP32 scratch for the per-split
// partial results.  Some callers have no way to allocate it: a host that binds
// only this C ABI and owns no device allocator, or an engine that reserves all
// free device memory at start-up so that any later cudaMalloc fails (and
// cudaMalloc/cudaFree may synchronize the device, which a decode loop cannot
// afford).  dak_attn_decode_noalloc serves them with scratch that lives in the
// library itself: a fixed array in device global memory, present on every GPU
// that loads the library, for the life of the process.
namespace dak {
namespace {
constexpr size_t kNoAllocScratchFloats = size_t(2) << 20;  // 8 MiB
static __device__ __align__(256) float g_attn_noalloc_scratch[kNoAllocScratchFloats];
constexpr int kNoAllocMaxDevices = 64;
// Where the array lives, per device, and in which context that was looked up:
// the address belongs to the context's copy of the library's module, so a
// different current context (another driver-API context, or the primary
// context created again after cudaDeviceReset) is looked up again.
struct NoAllocSlot {
  uint64_t ctx = 0;
  float *ptr = nullptr;
};
std::mutex g_noalloc_mu;
NoAllocSlot g_noalloc[kNoAllocMaxDevices];
}  // namespace
}  // namespace dak

extern "C" int dak_attn_decode_noalloc(const dak_attn_decode_args *args, void *stream) {
  using namespace dak;
  if (!args) return fail(DAK_ERR_INVALID_ARG, "args is null");
  int group, st;
  if ((st = common_checks(args->batch, args->num_q_heads, args->num_kv_heads, args->head_dim, args->split_size,
                          args->dtype, &group)))
    return st;
  if (args->seq_len <= 0) return fail(DAK_ERR_INVALID_ARG, "seq_len must be positive");
  const size_t splits = ((size_t)args->seq_len + (size_t)args->split_size - 1) / (size_t)args->split_size;
  dak_attn_decode_args a = *args;
  a.partial_o = nullptr;
  a.partial_ml = nullptr;
  if (splits > 1) {
    // Each factor is below 2^31 and the limit is 2^21, so bounding the running
    // product by the limit before every multiplication keeps it exact.
    const size_t per_row = (size_t)args->head_dim + 2;
    size_t need = per_row;
    const size_t factors[3] = {(size_t)args->batch, (size_t)args->num_q_heads, splits};
    for (size_t f : factors) {
      if (need > kNoAllocScratchFloats / f) {
        need = kNoAllocScratchFloats + 1;
        break;
      }
      need *= f;
    }
    if (need > kNoAllocScratchFloats)
      return fail(DAK_ERR_INVALID_ARG,
                  "dak_attn_decode_noalloc: batch x q_heads x splits x (head_dim + 2) exceeds its built-in "
                  "scratch of %zu floats (8 MiB); raise split_size or use dak_attn_decode",
                  kNoAllocScratchFloats);
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_status(e, "cudaGetDevice");
    if (dev < 0 || dev >= kNoAllocMaxDevices) return fail(DAK_ERR_UNSUPPORTED, "device %d out of range", dev);
    const uint64_t ctx = current_context_id();
    float *scratch;
    {
      // First call in this device's current context: look up where the array
      // lives there.  In host code the array's name is only a stand-in, never
      // a device address.
      std::lock_guard<std::mutex> lk(g_noalloc_mu);
      NoAllocSlot &slot = g_noalloc[dev];
      if (!slot.ptr || ctx == 0 || slot.ctx != ctx) {
        void *ptr = nullptr;
        e = cudaGetSymbolAddress(&ptr, g_attn_noalloc_scratch);
        if (e != cudaSuccess) return cuda_status(e, "cudaGetSymbolAddress(scratch)");
        slot.ptr = static_cast<float *>(ptr);
        slot.ctx = ctx ? ctx : current_context_id();
      }
      scratch = slot.ptr;
    }
    // Every partial (o, m, l) the merge reads is written earlier in the same
    // call, so the array needs no clearing between calls.
    const size_t rows = (size_t)args->batch * (size_t)args->num_q_heads * splits;
    a.partial_o = scratch;
    a.partial_ml = scratch + rows * (size_t)args->head_dim;
  }
  // With one split the kernel writes the output directly and uses no scratch.
  return dak_attn_decode(&a, stream);
}
