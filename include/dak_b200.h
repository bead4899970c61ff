/*
 * dak_b200.h - C ABI of the B200 (sm_100a) direct-access offloading kernels.
 *
 * Everything here is plain C: pointers, sizes and status codes, no torch or
 * pybind types.  A CUDA stream is passed as `void *` and must be a
 * `cudaStream_t` (NULL = legacy default stream).  No entry point allocates
 * device or host memory and none synchronizes the stream, so every launch can
 * be captured into a CUDA graph.
 *
 * Reference interfaces replaced (paths inside shouxulin/DirectAccessKernel):
 *   - src/torch_runtime.cu:120-468   pybind module `offload.runtime`
 *   - src/runtime.cu:9-16            print_device_name
 *   - include/task/utils.cuh:3-14    flush_l2_cache
 *   - opt_attention/csrc/opt_attention_ext.cpp:164-337 and
 *     opt_attention/csrc/opt_attention_kernel.cu:9-35   `opt_attention._C.decode`
 *
 * Every function returns DAK_OK (0) or a DAK_ERR_* code; dak_last_error_message()
 * gives the detail text of the calling thread's last failure.
 */
#ifndef DAK_B200_H
#define DAK_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define DAK_API __attribute__((visibility("default")))
#else
#define DAK_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---------------------------------------------------------------- status */
enum dak_status {
  DAK_OK = 0,
  DAK_ERR_INVALID_ARG = 1,  /* bad shape, stride, pointer or parameter       */
  DAK_ERR_UNSUPPORTED = 2,  /* valid but not implemented (dtype, head_dim...) */
  DAK_ERR_CUDA = 3,         /* a CUDA runtime call failed                     */
  DAK_ERR_DRIVER = 4,       /* a CUDA driver call failed (tensor-map encode)  */
  DAK_ERR_TIMEOUT = 5,      /* a bounded device-side wait gave up             */
  DAK_ERR_ALIGNMENT = 6,    /* pointer or stride breaks a 16-byte TMA rule    */
  DAK_ERR_NO_DEVICE = 7     /* no CUDA device visible                          */
};

/* Element types (match the dtypes accepted by torch_runtime.cu:87-107). */
enum dak_dtype {
  DAK_DTYPE_F16 = 0,
  DAK_DTYPE_BF16 = 1,
  DAK_DTYPE_F32 = 2,
  DAK_DTYPE_U8 = 3,
  DAK_DTYPE_I32 = 4,
  DAK_DTYPE_U32 = 5
};

/* Kernel opcodes, numbered as KERNEL_OPCODES in src/torch_runtime.cu:20-27. */
enum dak_opcode {
  DAK_OP_GEMV = 0,
  DAK_OP_GEMV_HORIZONTAL = 1,
  DAK_OP_GEMV_MULTICAST = 2,
  DAK_OP_GEMV_HORIZONTAL_MULTICAST = 3,
  DAK_OP_GEMV_MULTICAST_PREFILL = 4,
  DAK_OP_GEMV_HORIZONTAL_MULTICAST_PREFILL = 5
};

DAK_API const char *dak_strerror(int status);
/* Detail text of the calling thread's last failing call ("" if none). */
DAK_API const char *dak_last_error_message(void);

/* ------------------------------------------------------------- constants */
/* Module attributes NUM_SMS, MAX_COPY_SMS, BUFFER_SLOTS, TILE_N
 * (src/torch_runtime.cu:440-443; include/task/config.cuh:1-46). */
typedef struct dak_constants {
  int num_sms;       /* SMs of the current device (148 on B200)              */
  int max_copy_sms;  /* CTAs the linear kernels may occupy                    */
  int buffer_slots;  /* weight pipeline depth of the decode kernel           */
  int tile_n;        /* largest token count served by the CUDA-core kernel   */
  int tile_m;        /* output-feature granularity of the split (64)          */
  int tile_k;        /* K rows per pipeline stage                            */
  int mma_tile_m;    /* output features per tensor-core tile (128)           */
  int mma_max_tokens;/* tokens per tensor-core tile (UMMA N; 256); a launch  */
                     /* may cover up to twice as many as rows of tiles     */
  int abi_version;
} dak_constants;
DAK_API int dak_get_constants(dak_constants *out);

/* print_device_name (src/runtime.cu:9-16; torch_runtime.cu:419-422). */
DAK_API int dak_print_device_name(int device_id);

/* set_smem_size (src/torch_runtime.cu:373-417).  The sm_100a kernels size
 * their own shared memory, so this only validates the opcode and the request
 * against the device limit; it returns the size in effect, 0 on error. */
DAK_API size_t dak_set_smem_size(size_t smem_size, int opcode);

/* ------------------------------------------------------------ descriptors */
/* build_tma_desc (src/torch_runtime.cu:120-191).  Writes a DAK_DESC_BYTES
 * opaque descriptor of the tensor at `base` (a device pointer or a pinned,
 * mapped host pointer).  Arguments keep the reference's meaning: shape and
 * box in elements with the innermost dimension first, strides_bytes of
 * dimensions 1..rank-1 in bytes, swizzle 0/32/64/128.  The kernels rebuild
 * their own sm_100a tile maps from it, so the box is only checked. */
#define DAK_DESC_BYTES 128
DAK_API int dak_build_tma_desc(void *desc_out, const void *base, int dtype, int rank,
                       const int64_t *shape, const int64_t *strides_bytes,
                       const int64_t *box_dim, const int64_t *elem_strides,
                       int swizzle_bytes);

/* tensormap_replace_address (src/torch_runtime.cu:193-198). */
DAK_API int dak_tensormap_replace_address(void *desc, const void *new_base);

/* --------------------------------------------------- offloaded linear (a1-a3)
 * C[N, M] = B[N, K] * A[K, M] in the reference's naming: A is the transposed
 * weight (out features contiguous), B the activations (N tokens), C the
 * output.  FP32 accumulation, output written once (no pre-zeroed C needed).
 * num_copy_blocks / num_copy_host_blocks / *_sms_per_row keep their meaning
 * (CTAs in total, CTAs reading host rows, CTAs cooperating on one row tile);
 * 0 in num_copy_blocks selects the automatic B200 schedule.  smem_size is
 * accepted and ignored. */

/* gemv (src/torch_runtime.cu:201-221; include/task/gemv.cuh:372-405). */
DAK_API int dak_gemv(const void *a_desc, const void *b_desc, const void *c_desc, int M,
             int N, int K, int num_copy_blocks, int smem_size, int sms_per_row,
             void *stream);

/* gemv_horizontal (src/torch_runtime.cu:223-244; gemv.cuh:408-452): output
 * rows [0, h_M) come from the host-resident A, rows [h_M, h_M+d_M) from the
 * HBM-resident A. */
DAK_API int dak_gemv_horizontal(const void *a_desc_h, const void *a_desc_d,
                        const void *b_desc, const void *c_desc, int h_M,
                        int d_M, int N, int K, int num_copy_blocks,
                        int num_copy_host_blocks, int smem_size,
                        int h_sms_per_row, int d_sms_per_row, void *stream);

/* gemv_multicast / gemv_multicast_prefill (torch_runtime.cu:313-361;
 * gemv_multicast.cuh:185-376, 869-886).  Same contract as dak_gemv; served by
 * the tcgen05 kernel, which loads every weight tile once and uses no cluster
 * multicast. */
DAK_API int dak_gemv_multicast(const void *a_desc, const void *b_desc,
                       const void *c_desc, int M, int N, int K,
                       int num_copy_blocks, int smem_size, int sms_per_row,
                       void *stream);
DAK_API int dak_gemv_multicast_prefill(const void *a_desc, const void *b_desc,
                               const void *c_desc, int M, int N, int K,
                               int num_copy_blocks, int smem_size,
                               int sms_per_row, void *stream);

/* gemv_horizontal_multicast(_prefill) (torch_runtime.cu:247-311;
 * gemv_multicast.cuh:572-597, 889-914).  Same contract as dak_gemv_horizontal. */
DAK_API int dak_gemv_horizontal_multicast(const void *a_desc_h, const void *a_desc_d,
                                  const void *b_desc, const void *c_desc,
                                  int h_M, int d_M, int N, int K,
                                  int num_copy_blocks, int num_copy_host_blocks,
                                  int smem_size, int h_sms_per_row,
                                  int d_sms_per_row, void *stream);
DAK_API int dak_gemv_horizontal_multicast_prefill(
    const void *a_desc_h, const void *a_desc_d, const void *b_desc,
    const void *c_desc, int h_M, int d_M, int N, int K, int num_copy_blocks,
    int num_copy_host_blocks, int smem_size, int h_sms_per_row,
    int d_sms_per_row, void *stream);

/* Pointer-level form of the split linear that all the gemv* entry points
 * reduce to.  The weight is stored transposed, as the reference's
 * LinearHorizontal keeps it (app/python/layers/linearLayer.py:207-246):
 * w_host is [K, host_cols] with row stride ld_host elements, w_dev is
 * [K, dev_cols]; x is [ntok, K]; y is [ntok, *] and receives the host columns
 * at y[:, host_col_offset:...] and the device columns at y[:, dev_col_offset:...]. */
enum dak_linear_path {
  DAK_PATH_AUTO = 0,      /* CUDA-core for 1-2 tokens, tensor cores from 3    */
  DAK_PATH_CUDA_CORE = 1, /* FP32 FMA + warp-shuffle reduction, ntok <= 8     */
  DAK_PATH_TCGEN05 = 2    /* tcgen05.mma kind::f16, FP32 accumulators in TMEM */
};
typedef struct dak_linear_args {
  const void *w_host;
  int64_t host_cols, ld_host, host_col_offset;
  const void *w_dev;
  int64_t dev_cols, ld_dev, dev_col_offset;
  const void *x;
  int64_t ldx;
  void *y;
  int64_t ldy;
  int64_t ntok, K;
  int dtype;                  /* DAK_DTYPE_F16 or DAK_DTYPE_BF16          */
  int host_ctas, dev_ctas;    /* 0 = automatic                              */
  int host_ksplit, dev_ksplit;/* CTAs per output tile along K; 0 = automatic */
  int path;                   /* enum dak_linear_path                       */
} dak_linear_args;
DAK_API int dak_linear_split(const dak_linear_args *args, void *stream);

/* Gated linear (a SwiGLU MLP's gate and up projections with their activation):
 * the weight's output features alternate 16 gate rows and the 16 matching up
 * rows, and y[t, j] = silu(g_j) * u_j with g_j, u_j = x . W^T for the pair j
 * (feature c of the weight, with c % 32 < 16, pairs with c + 16 and writes y
 * column (c / 32) * 16 + c % 16).  Column offsets and counts of both tiers are
 * in the weight's feature space and must be multiples of 32; y needs
 * (offset + cols) / 2 columns.  The product is formed in FP32 from the FP32
 * accumulators and rounded once.  Runs on the tcgen05 kernel (any ntok) with
 * the same plans as dak_linear_split.  No kernel counterpart in the
 * reference: the vendored Llama MLP computes act_fn(gate_proj(x)) * up_proj(x)
 * in torch (app/python/llama/vanila_llama.py:188-209). */
DAK_API int dak_linear_split_glu(const dak_linear_args *args, void *stream);

/* Row-parallel linear with its all-reduce fused into the same kernel (no
 * reference counterpart; the reference has no multi-GPU path).  Every rank of a
 * tensor-parallel group calls it with the same shapes; y receives the sum over
 * ranks of x_rank . W_rank^T.  The tcgen05 kernel pushes each output tile's
 * 16-bit partial into every rank's receive buffer over peer memory (plain
 * stores), sets a per-CTA epoch flag on every rank, waits (bounded by
 * timeout_us; DAK_ERR_TIMEOUT in the device error word) for the same CTA of
 * every rank and sums the slots.  Buffers come from memory mapped into all
 * ranks (e.g. torch symmetric memory):
 *   buffers[r]: rank r's receive buffer, 2 x world x slot_elems 16-bit;
 *   flags[r]:   rank r's flags, 1024 x world uint32, zero before the first call;
 *   epoch/done: this rank's counters in device memory, zero before the first call.
 * slot_elems >= min(ntok, 256) x ldy.  Stream-ordered, graph-capturable, no
 * allocation; calls on one group must not overlap.
 * Multicast mode (own_f32 and mc_f32 given, e.g. on an NVSwitch box): each rank
 * stores its FP32 partials in its own buffer own_f32 (2 x slot_elems floats,
 * mapped into a multicast object whose address is mc_f32), publishes the flags,
 * and reads the sum over ranks with multimem.ld_reduce; buffers[] are unused. */
typedef struct dak_allreduce_args {
  int world, rank;
  void *buffers[8];
  uint32_t *flags[8];
  int64_t slot_elems;
  int *epoch, *done;
  int64_t timeout_us;
  float *own_f32, *mc_f32;
  int publish_only;   /* multicast mode only: store and publish; dak_rmsnorm_allreduce reduces */
} dak_allreduce_args;
DAK_API int dak_linear_split_allreduce(const dak_linear_args *args, const dak_allreduce_args *ar, void *stream);

/* The consumer side of publish-only mode (no reference counterpart): RMSNorm
 * whose input is the sum over ranks of the FP32 partials that the preceding
 * dak_linear_split_allreduce (publish_only = 1, same args) left in every rank's
 * buffer.  Waits, bounded, for every rank to publish the call; reads the sums
 * with multimem.ld_reduce; residual [rows, cols] (contiguous) is updated in
 * place to round16(round16(sum) + residual); out [rows, cols] receives the
 * normalised row.  ld is the row stride the linear used for its output.  Each
 * row is split over a cluster of 8 CTAs (cols <= 8192). */
DAK_API int dak_rmsnorm_allreduce(const dak_allreduce_args *ar, void *residual, const void *weight, void *out,
                                  int rows, int cols, int64_t ld, float eps, int dtype, void *stream);

/* flush_l2_cache (src/torch_runtime.cu:363-371; include/task/utils.cuh:3-14):
 * reads n floats of `dummy` past L2 and folds them into *sink. */
DAK_API int dak_flush_l2_cache(float *dummy, size_t n, float *sink, void *stream);

/* ------------------------------------------------ split-KV decode attention */
/* `opt_attention._C.decode` (opt_attention/csrc/opt_attention_ext.cpp:164-319).
 * One query token per sequence.  Rows b < host_size read key_host/value_host
 * (row b), the rest read key/value (row b - host_size), as
 * opt_attention_kernel.cuh:331-348 does.  K/V rows are [Hkv, S, D] with the
 * token stride equal to D.  num_q_heads may be a multiple of num_kv_heads
 * (GQA); the reference only has num_q_heads == num_kv_heads.  Partial results
 * of the split-KV pass go to the caller's scratch: partial_o holds
 * batch*num_q_heads*num_splits*head_dim floats and partial_ml
 * 2*batch*num_q_heads*num_splits floats, num_splits = ceil(S/split_size). */
typedef struct dak_attn_decode_args {
  const void *query;        /* [B, Hq, 1, D]                                */
  int64_t q_stride_b, q_stride_h;
  const void *key, *value;  /* device rows [B - host_size, Hkv, S, D]       */
  int64_t kv_stride_b, kv_stride_h;
  const void *key_host, *value_host; /* pinned rows [host_size, Hkv, S, D]  */
  int64_t kvh_stride_b, kvh_stride_h;
  const float *mask;        /* optional additive [B, 1, 1, S] FP32          */
  int64_t mask_stride_b;
  void *out;                /* [B, 1, Hq, D]                                */
  int64_t o_stride_b, o_stride_h;
  float *partial_o, *partial_ml;
  int batch, host_size, num_q_heads, num_kv_heads, head_dim, seq_len;
  int split_size;           /* tokens per split, multiple of 64            */
  float scaling;
  int dtype;                /* DAK_DTYPE_F16 or DAK_DTYPE_BF16             */
} dak_attn_decode_args;
DAK_API int dak_attn_decode(const dak_attn_decode_args *args, void *stream);

/* Allocation-free form of dak_attn_decode, with no counterpart in the
 * reference.  For callers that cannot allocate device memory: a host that binds
 * only this C ABI and has no device allocator of its own, or an engine that
 * has reserved all free device memory up front, so cudaMalloc would fail (and
 * cudaMalloc/cudaFree may synchronize the device).  The caller passes inputs
 * and outputs as for dak_attn_decode; args->partial_o and args->partial_ml are
 * ignored.  The split-KV partials go to an 8 MiB array inside the library,
 * held on every GPU that loads it until the process exits, so
 * batch * num_q_heads * ceil(seq_len / split_size) * (head_dim + 2) must not
 * exceed 2,097,152 floats; larger calls fail with DAK_ERR_INVALID_ARG.  A call
 * with one split (seq_len <= split_size) writes the output directly, uses no
 * scratch and has no such limit.  The first call in each CUDA context of a
 * device (the runtime's primary context, a context the host made current
 * through the driver API, or the primary context created again after
 * cudaDeviceReset) looks up the array's address in that context, so make that
 * first call before any stream capture.  All calls share the one array:
 * calls that can overlap on the GPU (different streams, different threads)
 * race on it and must be serialized by the caller.  The array keeps the last
 * call's contents; each call writes every partial it reads, so nothing needs
 * clearing.  Allocates nothing. */
DAK_API int dak_attn_decode_noalloc(const dak_attn_decode_args *args, void *stream);

/* Paged form: KV pages of page_size tokens live in two pools, one in HBM and
 * one in pinned host memory, both laid out [pages, Hkv, page_size, D].
 * block_table[b * bt_stride + j] names page j of sequence b: a value v >= 0 is
 * device page v, v < 0 is host page (-1 - v).  When either of dev_pages /
 * host_pages is > 0, both are the pools' page counts (0 = that pool is empty
 * or absent) and every entry is bounded by them: an entry past its pool reads
 * zeros and is recorded in the device error word (DAK_ERR_INVALID_ARG).  With
 * both 0 the entries are trusted.  No reference counterpart: the reference has
 * only the batch-split form above. */
typedef struct dak_attn_paged_args {
  const void *query;        /* [B, Hq, D]                                   */
  int64_t q_stride_b, q_stride_h;
  const void *k_pool_dev, *v_pool_dev;
  const void *k_pool_host, *v_pool_host;
  const int32_t *block_table;
  int64_t bt_stride;
  const int32_t *seq_lens;  /* [B] tokens per sequence                       */
  void *out;                /* [B, Hq, D]                                   */
  int64_t o_stride_b, o_stride_h;
  float *partial_o, *partial_ml;
  int batch, num_q_heads, num_kv_heads, head_dim, page_size, max_seq_len;
  int split_size;           /* tokens per split, multiple of page_size     */
  float scaling;
  int dtype;
  int64_t dev_pages, host_pages;  /* pages in each pool; both 0: unchecked */
} dak_attn_paged_args;
DAK_API int dak_attn_decode_paged(const dak_attn_paged_args *args, void *stream);

/* dak_attn_decode_paged with the split merge inside the attention kernel: the
 * last split of each (sequence, KV head) to finish merges every split's
 * partials, so no second kernel is launched.  merge_counters is caller-owned
 * device memory of batch * num_kv_heads int32, zero before the first call;
 * every completed call leaves it zero again.  Calls that share one counter
 * array must not overlap on the GPU.  Results are the same bits as
 * dak_attn_decode_paged's (the merge arithmetic is shared).  When
 * (num_q_heads / num_kv_heads) x splits exceeds about 8,000, the (m, l) pairs
 * do not fit the kernel's shared memory: the separate merge kernel runs and
 * the counters are not touched.  No reference
 * counterpart: the reference always launches a separate merge kernel
 * (opt_attention_kernel.cu:9-35). */
DAK_API int dak_attn_decode_paged_merged(const dak_attn_paged_args *args, int32_t *merge_counters, void *stream);

/* Appends one token per sequence to a tiered, paged KV cache: for sequence b
 * and KV head h, k_new[b, h, :] and v_new[b, h, :] go to slot
 * positions[b] % page_size of page block_table[b, positions[b] / page_size],
 * which is device page v (v >= 0) or host page -1 - v (v < 0), in the pool
 * layout of dak_attn_decode_paged ([pages, kv_heads, page_size, head_dim]).
 * Host pages are written by the GPU straight into pinned, mapped memory.
 * Replaces the reference's host-cache update (app/python/pinned_static_cache.py:
 * 47-107 with the synchronous copy at app/python/llama/vanila_llama.py:321-345).
 * Out-of-range entries are recorded in the device error word
 * (DAK_ERR_INVALID_ARG) and skipped.  No allocation; stream-ordered. */
typedef struct dak_kv_append_args {
  const void *k_new, *v_new;          /* [batch, kv_heads, head_dim]            */
  int64_t new_batch_stride, new_head_stride;  /* elements, multiples of 8        */
  void *k_pool_dev, *v_pool_dev;      /* device pools (or NULL)                 */
  int64_t dev_pages;
  void *k_pool_host, *v_pool_host;    /* pinned host pools (or NULL)            */
  int64_t host_pages;
  const int32_t *block_table;         /* [batch, table_stride]                  */
  int64_t table_stride;
  int max_pages;                      /* valid entries per table row            */
  const int32_t *positions;           /* [batch] token index to write           */
  int batch, kv_heads, head_dim, page_size;
  int dtype;
} dak_kv_append_args;
DAK_API int dak_kv_append_paged(const dak_kv_append_args *args, void *stream);

/* Rotary embedding and KV append of one decode step in one launch: for a
 * fused projection qkv [batch, (q_heads + 2 kv_heads) * head_dim] (row stride
 * ld), the q heads are rotated into q_out [batch, q_heads, head_dim] and the k
 * heads (rotated) and v heads are written into the paged pools exactly as
 * dak_rope_qk followed by dak_kv_append_paged would write them, positions and
 * pools taken from `kv` (kv->k_new / v_new are not read).  inv_freq holds
 * head_dim / 2 FP32 frequencies.  Out-of-range table entries are recorded in
 * the device error word and skipped.  No reference counterpart: the reference
 * applies rotary in torch (vanila_llama.py:212-246) and copies new K/V to its
 * host cache on the CPU (pinned_static_cache.py:47-107). */
DAK_API int dak_rope_kv_append(const void *qkv, int64_t ld, const float *inv_freq, void *q_out, int q_heads,
                               const dak_kv_append_args *kv, void *stream);

/* --------------------------------------------------- decode-layer helpers */
/* The element-wise steps of a Llama decode layer around the linears and the
 * attention.  No reference counterpart as kernels: the reference runs them as
 * torch ops in its vendored model (app/python/llama/vanila_llama.py:227-400);
 * these follow transformers' arithmetic op by op, roundings to 16 bit
 * included.  Stream-ordered, no allocation. */

/* out[r] = weight * round16(h * rsqrt(mean(h^2) + eps)), statistics in FP32, with
 * h = x[r] or, when residual is given, h = round16(x[r] + residual[r]), which is
 * also written to residual_out[r] (may alias x or residual).  x, residual and
 * residual_out share the row stride ld; out is [rows, cols] contiguous. */
DAK_API int dak_rmsnorm(const void *x, const void *residual, const void *weight, void *out, void *residual_out,
                        int rows, int cols, int64_t ld, float eps, int dtype, void *stream);

/* Rotary embedding (default rotary, rotate-half form) of the q and k heads of a
 * fused qkv row [q_heads | kv_heads | kv_heads] x head_dim with row stride ld:
 * angle = positions[b] * inv_freq[i] in FP32, cos/sin rounded to 16 bit; writes
 * q_out [batch, q_heads, head_dim], k_out and v_out [batch, kv_heads, head_dim]
 * (v copied unchanged). */
DAK_API int dak_rope_qk(const void *qkv, int64_t ld, const int32_t *positions, const float *inv_freq, void *q_out,
                        void *k_out, void *v_out, int batch, int q_heads, int kv_heads, int head_dim, int dtype,
                        void *stream);

/* out[r, c] = round16(silu(gate_up[r, c])) * gate_up[r, cols + c]; gate_up has
 * row stride ld (>= 2 cols), out is [rows, cols] contiguous. */
DAK_API int dak_silu_mul(const void *gate_up, int64_t ld, void *out, int rows, int cols, int dtype, void *stream);

/* ------------------------------------------------------------ diagnostics */
/* Reads (and with clear != 0 resets) the device-side error word that kernels
 * set when a bounded wait times out (DAK_ERR_TIMEOUT) or a block-table entry
 * is out of range (DAK_ERR_INVALID_ARG).  Synchronizes the current device. */
DAK_API int dak_device_status(int clear, int *status_out);

/* Failure-path self test (no reference counterpart): launches one CTA whose
 * mbarrier wait can never complete; the wait gives up after timeout_us
 * microseconds, records DAK_ERR_TIMEOUT in the device error word and the
 * kernel exits, leaving the context usable.  This is the path every kernel
 * takes when a copy or a peer never arrives. */
DAK_API int dak_selftest_wait_timeout(unsigned int timeout_us, void *stream);

/* Measurement helper: streams `bytes` of `src` (device or pinned host memory)
 * through shared memory with TMA bulk copies on `ctas` CTAs, each keeping
 * `stages` copies of `chunk_bytes` in flight; folds a checksum into *sink. */
DAK_API int dak_probe_stream_read(const void *src, size_t bytes, int ctas, int stages,
                          int chunk_bytes, uint32_t *sink, void *stream);

#ifdef __cplusplus
}
#endif
#endif /* DAK_B200_H */
