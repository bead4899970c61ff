// dak_kv.cu - the writer side of the tiered, paged KV cache.
//
// Each decode step appends one token's K and V per (sequence, KV head) to the
// page the block table names for that token: a device page in HBM or a host
// page in pinned, mapped host memory.  The GPU writes host pages directly over
// the host link; nothing is staged and nothing waits on the CPU.
//
// Replaces the reference's host-cache update (app/python/pinned_static_cache.py:
// 47-107, fed by `.to("cpu").pin_memory()` in app/python/llama/vanila_llama.py:
// 321-345), which copies the new K/V to the host synchronously and scatters them
// with the CPU every step.
#include <cstring>

#include "dak_common.cuh"
#include "dak_host.h"

namespace dak {
namespace {

struct KvAppendParams {
  const uint8_t *k_new, *v_new;
  long long new_bs, new_hs;            // bytes
  uint8_t *pool[2][2];                 // [k/v][device/host]
  long long pages[2];                  // device, host
  long long page_bytes, head_bytes;    // bytes of one page / one head's slab in a page
  const int32_t *table;
  long long table_stride;              // entries
  const int32_t *positions;
  int max_pages;                       // table entries per sequence
  int kv_heads, row_bytes, page_size;
  int *status;
  int pdl;                             // launched with programmatic stream serialization
};

// Page slot of token positions[b], KV head h, in pool tier *tier (0 device,
// 1 host): byte offset into that tier's pools, or -1 for an out-of-range
// position or table entry (recorded in the status word by the caller).
__device__ __forceinline__ long long kv_slot(const KvAppendParams &p, int b, int h, int *tier) {
  const int pos = p.positions[b];
  const int page = pos / p.page_size;
  if (pos < 0 || page >= p.max_pages) return -1;
  const int entry = p.table[(long long)b * p.table_stride + page];
  *tier = entry < 0 ? 1 : 0;
  const long long idx = entry < 0 ? -1ll - entry : entry;
  if (idx >= p.pages[*tier] || p.pool[0][*tier] == nullptr) return -1;
  return idx * p.page_bytes + h * p.head_bytes + (long long)(pos - page * p.page_size) * p.row_bytes;
}

// One warp per (sequence, KV head): lanes split the K row and the V row into
// 16-byte pieces.  Out-of-range table entries or positions are recorded in the
// status word and skipped, never written.
__global__ void __launch_bounds__(32) kv_append_kernel(const __grid_constant__ KvAppendParams p) {
  pdl_enter(p.pdl);
  const int b = blockIdx.x / p.kv_heads;
  const int h = blockIdx.x - b * p.kv_heads;
  int tier = 0;
  const long long dst_off = kv_slot(p, b, h, &tier);
  if (dst_off < 0) {
    if (threadIdx.x == 0) atomicCAS(p.status, 0, DAK_ERR_INVALID_ARG);
    return;
  }
  const long long src_off = b * p.new_bs + h * p.new_hs;
  const int pieces = p.row_bytes / 16;
  for (int i = threadIdx.x; i < 2 * pieces; i += 32) {
    const int kv = i >= pieces ? 1 : 0;
    const int piece = i - kv * pieces;
    const uint8_t *src = (kv ? p.v_new : p.k_new) + src_off + piece * 16;
    uint8_t *dst = p.pool[kv][tier] + dst_off + piece * 16;
    *reinterpret_cast<uint4 *>(dst) = *reinterpret_cast<const uint4 *>(src);
  }
  // Host pages are read back over the host link by the next kernels of the
  // stream; make the writes visible system-wide before this grid completes.
  if (tier == 1) __threadfence_system();
}

struct RopeAppendParams {
  KvAppendParams kv;      // pools, block table and positions; k_new / v_new unused
  const void *qkv;        // [batch, (q_heads + 2 kv_heads) * head_dim], row stride ld
  long long ld;
  const float *inv_freq;  // [head_dim / 2]
  void *q_out;            // [batch, q_heads, head_dim]
  int q_heads, head_dim;
};

// Rotary q/k plus the KV append of the new token in one launch: one CTA per
// (sequence, head) of q, k and v, head_dim / 2 threads.  q heads are rotated
// into q_out; k heads are rotated and v heads copied straight into the page
// slot the block table names for the token, in HBM or pinned host memory.
// The rotation is rope_qk_kernel's; the slot is kv_append_kernel's.
template <typename T>
__global__ void rope_kv_append_kernel(const __grid_constant__ RopeAppendParams p) {
  pdl_enter(p.kv.pdl);
  const int hkv = p.kv.kv_heads;
  const int heads = p.q_heads + 2 * hkv;
  const int b = blockIdx.x / heads;
  const int hh = blockIdx.x - b * heads;
  const int half = p.head_dim / 2;
  const int i = threadIdx.x;
  const uint16_t *src = static_cast<const uint16_t *>(p.qkv) + (long long)b * p.ld + (long long)hh * p.head_dim;
  uint16_t *dst;
  int tier = 0;
  if (hh < p.q_heads) {
    dst = static_cast<uint16_t *>(p.q_out) + ((long long)b * p.q_heads + hh) * p.head_dim;
  } else {
    const int isv = hh >= p.q_heads + hkv ? 1 : 0;
    const long long off = kv_slot(p.kv, b, hh - p.q_heads - isv * hkv, &tier);
    if (off < 0) {
      if (i == 0) atomicCAS(p.kv.status, 0, DAK_ERR_INVALID_ARG);
      return;
    }
    dst = reinterpret_cast<uint16_t *>(p.kv.pool[isv][tier] + off);
  }
  if (i < half) {
    if (hh < p.q_heads + hkv) {
      float o1, o2;
      rope_pair<T>(Elem<T>::to_float(src[i]), Elem<T>::to_float(src[i + half]),
                   (float)p.kv.positions[b] * p.inv_freq[i], o1, o2);
      dst[i] = Elem<T>::from_float(o1);
      dst[i + half] = Elem<T>::from_float(o2);
    } else {
      dst[i] = src[i];
      dst[i + half] = src[i + half];
    }
  }
  // Host pages are read back over the host link by the next kernels of the
  // stream; make the writes visible system-wide before this grid completes.
  if (tier == 1) __threadfence_system();
}

// Checks of the pools, table and positions shared by both entry points, and
// the kernel parameters they give.  `need_new`: k_new / v_new are read.
int kv_params(const dak_kv_append_args *a, bool need_new, KvAppendParams *out) {
  if (!a) return fail(DAK_ERR_INVALID_ARG, "args is null");
  if (a->dtype != DAK_DTYPE_F16 && a->dtype != DAK_DTYPE_BF16)
    return fail(DAK_ERR_UNSUPPORTED, "KV append supports float16 and bfloat16");
  if (a->batch <= 0 || a->kv_heads <= 0 || a->head_dim <= 0 || a->page_size <= 0 || a->max_pages <= 0)
    return fail(DAK_ERR_INVALID_ARG, "batch, kv_heads, head_dim, page_size and max_pages must be positive");
  if ((a->head_dim * 2) % 16 != 0) return fail(DAK_ERR_ALIGNMENT, "head_dim must be a multiple of 8");
  if ((need_new && (!a->k_new || !a->v_new)) || !a->block_table || !a->positions)
    return fail(DAK_ERR_INVALID_ARG, need_new ? "k_new, v_new, block_table and positions are required"
                                              : "block_table and positions are required");
  if (a->table_stride < a->max_pages) return fail(DAK_ERR_INVALID_ARG, "table_stride below max_pages");
  if ((a->dev_pages > 0) != (a->k_pool_dev != nullptr && a->v_pool_dev != nullptr) ||
      (a->host_pages > 0) != (a->k_pool_host != nullptr && a->v_pool_host != nullptr))
    return fail(DAK_ERR_INVALID_ARG, "each tier needs both pools and a positive page count, or neither");
  if (a->dev_pages <= 0 && a->host_pages <= 0) return fail(DAK_ERR_INVALID_ARG, "no KV pool given");
  if (need_new && ((a->new_batch_stride % 8) || (a->new_head_stride % 8)))
    return fail(DAK_ERR_ALIGNMENT, "k_new/v_new strides must be multiples of 8 elements");
  const void *ptrs[6] = {need_new ? a->k_new : nullptr, need_new ? a->v_new : nullptr, a->k_pool_dev,
                         a->v_pool_dev, a->k_pool_host, a->v_pool_host};
  for (const void *q : ptrs) {
    if (q && (reinterpret_cast<uintptr_t>(q) & 15u)) return fail(DAK_ERR_ALIGNMENT, "all buffers must be 16-byte aligned");
    if (q) {
      int st = check_gpu_accessible(q, "KV buffer");
      if (st) return st;
    }
  }
  KvAppendParams &p = *out;
  std::memset(&p, 0, sizeof(p));
  p.k_new = static_cast<const uint8_t *>(a->k_new);
  p.v_new = static_cast<const uint8_t *>(a->v_new);
  p.new_bs = a->new_batch_stride * 2;
  p.new_hs = a->new_head_stride * 2;
  p.pool[0][0] = static_cast<uint8_t *>(a->k_pool_dev);
  p.pool[1][0] = static_cast<uint8_t *>(a->v_pool_dev);
  p.pool[0][1] = static_cast<uint8_t *>(a->k_pool_host);
  p.pool[1][1] = static_cast<uint8_t *>(a->v_pool_host);
  p.pages[0] = a->dev_pages > 0 ? a->dev_pages : 0;
  p.pages[1] = a->host_pages > 0 ? a->host_pages : 0;
  p.row_bytes = a->head_dim * 2;
  p.head_bytes = (long long)a->page_size * p.row_bytes;
  p.page_bytes = p.head_bytes * a->kv_heads;
  p.table = a->block_table;
  p.table_stride = a->table_stride;
  p.positions = a->positions;
  p.max_pages = a->max_pages;
  p.kv_heads = a->kv_heads;
  p.page_size = a->page_size;
  p.status = device_status_word();
  if (!p.status) return fail(DAK_ERR_CUDA, "no device status word");
  p.pdl = decode_pdl_enabled() ? 1 : 0;
  return DAK_OK;
}

}  // namespace
}  // namespace dak

extern "C" int dak_rope_kv_append(const void *qkv, int64_t ld, const float *inv_freq, void *q_out, int q_heads,
                                  const dak_kv_append_args *kv, void *stream) {
  using namespace dak;
  RopeAppendParams p;
  std::memset(&p, 0, sizeof(p));
  int st = kv_params(kv, false, &p.kv);
  if (st) return st;
  if (!qkv || !inv_freq || !q_out || q_heads <= 0)
    return fail(DAK_ERR_INVALID_ARG, "rope_kv_append: qkv, inv_freq, q_out and q_heads > 0 are required");
  if (kv->head_dim % 2 || kv->head_dim > 1024)
    return fail(DAK_ERR_INVALID_ARG, "rope_kv_append: head_dim must be even and at most 1024");
  if (ld < (int64_t)(q_heads + 2 * kv->kv_heads) * kv->head_dim)
    return fail(DAK_ERR_INVALID_ARG, "rope_kv_append: qkv row stride below (q_heads + 2 kv_heads) x head_dim");
  p.qkv = qkv;
  p.ld = ld;
  p.inv_freq = inv_freq;
  p.q_out = q_out;
  p.q_heads = q_heads;
  p.head_dim = kv->head_dim;
  const int grid = kv->batch * (q_heads + 2 * kv->kv_heads);
  const int threads = ((kv->head_dim / 2 + 31) / 32) * 32;
  auto s = static_cast<cudaStream_t>(stream);
  const cudaError_t e = kv->dtype == DAK_DTYPE_F16
                            ? launch_ex(rope_kv_append_kernel<__half>, dim3(grid), dim3(threads), 0, s, 1,
                                        p.kv.pdl != 0, p)
                            : launch_ex(rope_kv_append_kernel<__nv_bfloat16>, dim3(grid), dim3(threads), 0, s, 1,
                                        p.kv.pdl != 0, p);
  return cuda_status(e, "rope_kv_append launch");
}

extern "C" int dak_kv_append_paged(const dak_kv_append_args *a, void *stream) {
  using namespace dak;
  KvAppendParams p;
  int st = kv_params(a, true, &p);
  if (st) return st;
  const cudaError_t e = launch_ex(kv_append_kernel, dim3(a->batch * a->kv_heads), dim3(32), 0,
                                  static_cast<cudaStream_t>(stream), 1, p.pdl != 0, p);
  return cuda_status(e, "KV append launch");
}
