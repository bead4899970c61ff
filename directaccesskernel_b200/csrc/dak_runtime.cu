// dak_runtime.cu - the C ABI of libdak_b200.so (include/dak_b200.h) for the
// offloaded linear layers: descriptors, tile-map encoding, scheduling of the
// host and device tiers, launches, L2 flush, the device error word and the
// host-link read probe.
//
// Reference: src/torch_runtime.cu (pybind module `offload.runtime`),
// src/runtime.cu, include/task/utils.cuh.
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <set>
#include <string>
#include <unordered_map>
#include <utility>

#include "dak_common.cuh"
#include "dak_host.h"
#include "dak_linear.cuh"

// Device error word written by every kernel's bounded waits.
__device__ int g_dak_status;

namespace dak {

// ------------------------------------------------------------------ errors
static thread_local char t_last_error[512];

int fail(int code, const char *fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(t_last_error, sizeof(t_last_error), fmt, ap);
  va_end(ap);
  return code;
}

int cuda_status(cudaError_t e, const char *what) {
  if (e == cudaSuccess) return DAK_OK;
  if (e == cudaErrorNoDevice || e == cudaErrorInsufficientDriver)
    return fail(DAK_ERR_NO_DEVICE, "%s: %s", what, cudaGetErrorString(e));
  return fail(DAK_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

// -------------------------------------------------------- per-device state
// Identity of the CUDA context that is current on the calling thread (the
// runtime's primary context, or one that a C-ABI host made current through
// the driver API), or 0 when none is.  cuCtxGetId numbers contexts uniquely
// for the life of the process, so a context created after cudaDeviceReset
// gets a new identity even if its handle is reused.  Device addresses of the
// library's `__device__` arrays and kernel attributes belong to one context,
// so the state below is set up again whenever the current context's identity
// differs from the one it was set up in.
uint64_t current_context_id() {
  using CtxGetCurrent = CUresult (*)(CUcontext *);
  using CtxGetId = CUresult (*)(CUcontext, unsigned long long *);
  static const std::pair<CtxGetCurrent, CtxGetId> fn = [] {
    auto entry = [](const char *name) -> void * {
      void *p = nullptr;
      cudaDriverEntryPointQueryResult q;
      if (cudaGetDriverEntryPointByVersion(name, &p, 12000, cudaEnableDefault, &q) != cudaSuccess ||
          q != cudaDriverEntryPointSuccess)
        return nullptr;
      return p;
    };
    return std::make_pair(reinterpret_cast<CtxGetCurrent>(entry("cuCtxGetCurrent")),
                          reinterpret_cast<CtxGetId>(entry("cuCtxGetId")));
  }();
  CUcontext ctx = nullptr;
  unsigned long long id = 0;
  if (!fn.first || !fn.second || fn.first(&ctx) != CUDA_SUCCESS || !ctx || fn.second(ctx, &id) != CUDA_SUCCESS)
    return 0;
  return (uint64_t)id + 1;  // never 0 for a live context
}

namespace {
constexpr int kMaxDevices = 64;

struct DeviceInfo {
  bool ready = false;
  uint64_t ctx = 0;  // identity of the context the entry was set up in
  int num_sms = 0;
  int max_smem_optin = 0;
  int *status = nullptr;
};
std::mutex g_dev_mu;
DeviceInfo g_dev[kMaxDevices];

int current_device(int *dev) {
  cudaError_t e = cudaGetDevice(dev);
  if (e != cudaSuccess) return cuda_status(e, "cudaGetDevice");
  if (*dev < 0 || *dev >= kMaxDevices) return fail(DAK_ERR_UNSUPPORTED, "device %d out of range", *dev);
  return DAK_OK;
}

int device_info(DeviceInfo **out) {
  int dev;
  int st = current_device(&dev);
  if (st) return st;
  const uint64_t ctx = current_context_id();
  std::lock_guard<std::mutex> lk(g_dev_mu);
  DeviceInfo &d = g_dev[dev];
  // No context yet means the runtime has not made one current: the symbol
  // lookup below creates it, and the entry records it afterwards.
  if (!d.ready || ctx == 0 || ctx != d.ctx) {
    d.ready = false;
    cudaError_t e = cudaDeviceGetAttribute(&d.num_sms, cudaDevAttrMultiProcessorCount, dev);
    if (e == cudaSuccess)
      e = cudaDeviceGetAttribute(&d.max_smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    if (e == cudaSuccess) e = cudaGetSymbolAddress(reinterpret_cast<void **>(&d.status), g_dak_status);
    if (e != cudaSuccess) return cuda_status(e, "device query");
    d.ctx = ctx ? ctx : current_context_id();
    d.ready = true;
  }
  *out = &d;
  return DAK_OK;
}
}  // namespace

int *device_status_word() {
  DeviceInfo *d = nullptr;
  return device_info(&d) == DAK_OK ? d->status : nullptr;
}

cudaError_t prepare_kernel_attributes(const void *kern) {
  static std::mutex mu;
  static std::set<std::pair<uint64_t, const void *>> done;  // (context identity, kernel)
  DeviceInfo *d = nullptr;
  if (device_info(&d) != DAK_OK) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lk(mu);
  if (d->ctx && done.count({d->ctx, kern})) return cudaSuccess;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, d->max_smem_optin);
  if (e == cudaSuccess) e = cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
  if (e == cudaSuccess && d->ctx) done.insert({d->ctx, kern});
  return e;
}

// A kernel may only be pointed at memory of the current device or at pinned
// (page-locked, mapped) host memory; anything else would fault the GPU.
int check_gpu_accessible(const void *p, const char *what) {
  cudaPointerAttributes attr;
  cudaError_t e = cudaPointerGetAttributes(&attr, p);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return fail(DAK_ERR_INVALID_ARG, "%s: cannot query the pointer (%s)", what, cudaGetErrorString(e));
  }
  if (attr.type == cudaMemoryTypeHost) return DAK_OK;
  if (attr.type == cudaMemoryTypeDevice || attr.type == cudaMemoryTypeManaged) {
    int dev = -1;
    cudaGetDevice(&dev);
    if (attr.type == cudaMemoryTypeDevice && attr.device != dev)
      return fail(DAK_ERR_INVALID_ARG, "%s lives on device %d, not the current device %d", what, attr.device, dev);
    return DAK_OK;
  }
  return fail(DAK_ERR_INVALID_ARG, "%s must be device memory or pinned host memory (pageable memory given)", what);
}

// ------------------------------------------------------ tile-map encoding
namespace {
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;

int encode_fn(PFN_cuTensorMapEncodeTiled_v12000 *fn) {
  std::call_once(g_encode_once, []() {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault,
                                         &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  if (!g_encode) return fail(DAK_ERR_DRIVER, "cuTensorMapEncodeTiled entry point unavailable");
  *fn = g_encode;
  return DAK_OK;
}

struct MapKey {
  uint64_t base, dim0, dim1, stride1;
  uint32_t box0, box1, dtype, swizzle;
  bool operator==(const MapKey &o) const { return std::memcmp(this, &o, sizeof(MapKey)) == 0; }
};
struct MapKeyHash {
  size_t operator()(const MapKey &k) const {
    const uint64_t *w = reinterpret_cast<const uint64_t *>(&k);
    uint64_t h = 1469598103934665603ull;
    for (size_t i = 0; i < sizeof(MapKey) / 8; ++i) h = (h ^ w[i]) * 1099511628211ull;
    return (size_t)h;
  }
};
std::mutex g_map_mu;
std::unordered_map<MapKey, CUtensorMap, MapKeyHash> g_map_cache;

CUtensorMapDataType cu_dtype(int dtype) {
  switch (dtype) {
    case DAK_DTYPE_F16: return CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    case DAK_DTYPE_BF16: return CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
    case DAK_DTYPE_F32: return CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
    case DAK_DTYPE_U8: return CU_TENSOR_MAP_DATA_TYPE_UINT8;
    case DAK_DTYPE_I32: return CU_TENSOR_MAP_DATA_TYPE_INT32;
    default: return CU_TENSOR_MAP_DATA_TYPE_UINT32;
  }
}

// 2-D tile map over a row-major matrix [rows, cols] with row stride ld
// elements; box {box_cols, box_rows}; zero fill out of bounds.
int tile_map_2d(CUtensorMap *out, const void *base, int dtype, int64_t rows, int64_t cols,
                int64_t ld, int box_cols, int box_rows, int swizzle_bytes) {
  const MapKey key{reinterpret_cast<uint64_t>(base), (uint64_t)cols, (uint64_t)rows,
                   (uint64_t)ld * 2u, (uint32_t)box_cols, (uint32_t)box_rows, (uint32_t)dtype,
                   (uint32_t)swizzle_bytes};
  {
    std::lock_guard<std::mutex> lk(g_map_mu);
    auto it = g_map_cache.find(key);
    if (it != g_map_cache.end()) {
      *out = it->second;
      return DAK_OK;
    }
  }
  int st = check_gpu_accessible(base, "matrix");
  if (st) return st;
  PFN_cuTensorMapEncodeTiled_v12000 fn;
  st = encode_fn(&fn);
  if (st) return st;
  const cuuint64_t gdim[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  const cuuint64_t gstride[1] = {(cuuint64_t)ld * 2u};
  const cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
  const cuuint32_t estride[2] = {1, 1};
  const CUtensorMapSwizzle swz =
      swizzle_bytes == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE;
  CUresult r = fn(out, cu_dtype(dtype), 2, const_cast<void *>(base), gdim, gstride, box, estride,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(DAK_ERR_DRIVER, "cuTensorMapEncodeTiled failed (%d) for [%lld x %lld] ld %lld", (int)r,
                (long long)rows, (long long)cols, (long long)ld);
  std::lock_guard<std::mutex> lk(g_map_mu);
  if (g_map_cache.size() > 4096) g_map_cache.clear();
  g_map_cache.emplace(key, *out);
  return DAK_OK;
}
}  // namespace

// --------------------------------------------------------- descriptor blob
namespace {
constexpr uint32_t kDescMagic = 0x444B4144u;  // "DAKD"

struct DescBlob {
  uint32_t magic;
  uint16_t version;
  uint8_t dtype;
  uint8_t rank;
  uint64_t base;
  uint64_t shape[5];
  uint64_t strides[4];
  uint16_t box[5];
  uint8_t elem_strides[5];
  uint8_t swizzle;
  uint8_t reserved[24];
};
static_assert(sizeof(DescBlob) == DAK_DESC_BYTES, "descriptor blob must be 128 bytes");

int elem_size(int dtype) {
  switch (dtype) {
    case DAK_DTYPE_F16:
    case DAK_DTYPE_BF16: return 2;
    case DAK_DTYPE_U8: return 1;
    case DAK_DTYPE_F32:
    case DAK_DTYPE_I32:
    case DAK_DTYPE_U32: return 4;
    default: return 0;
  }
}

struct MatView {
  const void *base;
  int64_t rows, cols, ld;  // row-major, cols contiguous
  int dtype;
};

// Recovers the row-major matrix a descriptor describes.  Accepts the forms the
// reference's helpers build (app/python/utils.py:48-145): plain 2-D
// [cols, rows]; the 4-D blocked MN form [64, 8, cols/64, rows/8]; the 3-D
// K-major activation form [64, rows, cols/64]; a trailing batch dimension that
// continues the rows.
int desc_to_matrix(const void *blob, const char *what, MatView *out) {
  if (!blob) return fail(DAK_ERR_INVALID_ARG, "%s descriptor is null", what);
  DescBlob d;
  std::memcpy(&d, blob, sizeof(d));
  if (d.magic != kDescMagic) return fail(DAK_ERR_INVALID_ARG, "%s is not a DAK descriptor", what);
  const int es = elem_size(d.dtype);
  const uint64_t *sh = d.shape;
  const uint64_t *st = d.strides;
  MatView m{reinterpret_cast<const void *>(d.base), 0, 0, 0, d.dtype};
  switch (d.rank) {
    case 1:
      m.cols = (int64_t)sh[0];
      m.rows = 1;
      m.ld = m.cols;
      break;
    case 2:
      m.cols = (int64_t)sh[0];
      m.rows = (int64_t)sh[1];
      m.ld = (int64_t)(st[0] / es);
      break;
    case 3:
      if (st[1] == sh[0] * (uint64_t)es) {  // [blk, rows, cols/blk] K-major activation form
        m.cols = (int64_t)(sh[0] * sh[2]);
        m.rows = (int64_t)sh[1];
        m.ld = (int64_t)(st[0] / es);
      } else if (st[1] == st[0] * sh[1]) {  // [cols, rows, batch]
        m.cols = (int64_t)sh[0];
        m.rows = (int64_t)(sh[1] * sh[2]);
        m.ld = (int64_t)(st[0] / es);
      } else {
        return fail(DAK_ERR_INVALID_ARG, "%s: unsupported rank-3 descriptor layout", what);
      }
      break;
    case 4:
      if (st[1] == sh[0] * (uint64_t)es && st[2] == st[0] * sh[1]) {  // [blkM, blkK, M/blkM, K/blkK]
        m.cols = (int64_t)(sh[0] * sh[2]);
        m.rows = (int64_t)(sh[1] * sh[3]);
        m.ld = (int64_t)(st[0] / es);
      } else {
        return fail(DAK_ERR_INVALID_ARG, "%s: unsupported rank-4 descriptor layout", what);
      }
      break;
    default:
      return fail(DAK_ERR_INVALID_ARG, "%s: unsupported descriptor rank %d", what, (int)d.rank);
  }
  if (m.ld < m.cols) return fail(DAK_ERR_INVALID_ARG, "%s: row stride below row length", what);
  *out = m;
  return DAK_OK;
}
}  // namespace

bool decode_pdl_enabled() {
  static const bool on = [] {
    const char *off = getenv("DAK_B200_NO_PDL");
    return !(off && off[0] && off[0] != '0');
  }();
  return on;
}

// ---------------------------------------------------------- the split linear
namespace {
constexpr int kAutoHostCtas = 8;  // two CTAs with 4 x 32 KB in flight already saturate PCIe Gen5
constexpr int kMinSplitRows = 1536;  // K rows each CTA of a split keeps at least (12 stages)
constexpr int kCoreMaxKsplit = 8;
constexpr int kMmaMaxKsplitHost = 4;

int pow2_floor(int v) {
  int p = 1;
  while (p * 2 <= v) p *= 2;
  return p;
}

struct TierPlan {
  int ctas = 0;    // working CTAs (multiple of ksplit)
  int ksplit = 1;
};

// Automatic plan for one tier: `budget` CTAs, `tiles` output tiles, `nkb` K blocks.
TierPlan auto_plan(int budget, int tiles, int nkb, int max_ks) {
  TierPlan t;
  if (tiles <= 0 || budget <= 0) return t;
  int ks = 1;
  while (ks * 2 <= max_ks && tiles * ks * 2 <= budget && ks * 2 <= nkb / 2) ks *= 2;
  t.ksplit = ks;
  t.ctas = std::min(budget / ks, tiles) * ks;
  if (t.ctas == 0) {
    t.ksplit = 1;
    t.ctas = std::min(budget, tiles);
  }
  return t;
}

// User plan (reference arguments): `ctas` CTAs, `spr` CTAs per row tile.
TierPlan user_plan(int ctas, int spr, int tiles, int nkb, int max_ks) {
  TierPlan t;
  if (tiles <= 0 || ctas <= 0) return t;
  int ks = std::max(1, std::min(spr, max_ks));
  ks = std::min(ks, std::max(1, nkb));
  if (ks > 1) ks = pow2_floor(ks);
  t.ksplit = ks;
  t.ctas = std::max(ks, (ctas / ks) * ks);
  return t;
}

// DAK_B200_TRACE_PLAN=1 prints every launch plan of the linear kernels to stderr.
bool trace_plans() {
  static const bool on = [] {
    const char *v = getenv("DAK_B200_TRACE_PLAN");
    return v && v[0] && v[0] != '0';
  }();
  return on;
}

// Programmatic dependent launch of the linear kernels; DAK_B200_NO_PDL=1 turns it off.
bool pdl_enabled() {
  static const bool on = [] {
    const char *v = getenv("DAK_B200_NO_PDL");
    return !(v && v[0] && v[0] != '0');
  }();
  return on;
}

// CTAs of one launch that can be resident at once, for a kernel variant and
// cluster size (cached occupancy query).
int max_resident_ctas(bool mma, int tmpl, int dtype, int cluster, size_t smem, int num_sms) {
  static std::mutex mu;
  static std::unordered_map<uint64_t, int> cache;
  int dev = 0;
  cudaGetDevice(&dev);
  const uint64_t key = ((uint64_t)dev << 56) | ((uint64_t)mma << 55) | ((uint64_t)(dtype & 7) << 52) |
                       ((uint64_t)(tmpl & 0x3FF) << 40) | ((uint64_t)(cluster & 0xFF) << 32) | (uint64_t)smem;
  {
    std::lock_guard<std::mutex> lk(mu);
    auto it = cache.find(key);
    if (it != cache.end()) return it->second;
  }
  LinearParams probe;
  std::memset(&probe, 0, sizeof(probe));
  probe.pdl = pdl_enabled() ? 1 : 0;
  int clusters = 0;
  cudaError_t e = mma ? launch_linear_mma(probe, tmpl, dtype, 0, cluster, smem, nullptr, &clusters)
                      : launch_linear_core(probe, tmpl, dtype, 0, cluster, smem, nullptr, &clusters);
  int ctas = (e == cudaSuccess && clusters > 0) ? clusters * cluster : 0;
  if (e != cudaSuccess) cudaGetLastError();
  if (ctas > num_sms) ctas = num_sms;  // one CTA per SM: shared memory allows no more
  std::lock_guard<std::mutex> lk(mu);
  cache[key] = ctas;
  return ctas;
}

int check_ptr16(const void *p, const char *what) {
  if ((reinterpret_cast<uintptr_t>(p) & 15u) != 0)
    return fail(DAK_ERR_ALIGNMENT, "%s must be 16-byte aligned", what);
  return DAK_OK;
}

// One chunk of 257..512 tokens on the wide kernel.  Every CTA walks an even
// share of whole 64-feature boxes of its tier.  The host tier gets up to
// kWideHostCtas CTAs: each keeps two 16 KB weight stages in flight, so 32 of
// them hold about 1 MB in flight, several times what the host link needs.  The
// device tier, bound by tensor-core work at this batch size, gets the rest of
// the SMs (one CTA per SM: the kernel takes about 161 KB of shared memory).
constexpr int kWideHostCtas = 32;

// With pair_groups > 0 (an HBM-only layer), the paired mode instead: that many
// CTAs per 256-token row of the chunk, each applying its row to two
// 128-feature tiles at a time.
int run_linear_wide_chunk(const dak_linear_args *a, const DeviceInfo *dev, int64_t t0, int64_t nt,
                          cudaStream_t stream, int pair_groups = 0) {
  const bool pair = pair_groups > 0;
  const int boxes_h = (int)((a->host_cols + kBoxCols - 1) / kBoxCols);
  const int boxes_d = (int)((a->dev_cols + kBoxCols - 1) / kBoxCols);
  if (pair && boxes_h > 0) return fail(DAK_ERR_INVALID_ARG, "paired wide linear: the layer has host rows");
  const int hc = boxes_h > 0 ? std::max(1, std::min({kWideHostCtas, boxes_h, dev->num_sms / 2})) : 0;
  const int dc = pair ? pair_groups : boxes_d > 0 ? std::max(1, std::min(dev->num_sms - hc, boxes_d)) : 0;
  const int64_t tiers_cols[2] = {a->host_cols, a->dev_cols};
  const void *tiers_w[2] = {a->w_host, a->w_dev};
  const int64_t tiers_ld[2] = {a->ld_host, a->ld_dev};
  const int64_t tiers_off[2] = {a->host_col_offset, a->dev_col_offset};
  const int ctas[2] = {hc, dc};
  LinearParams p;
  std::memset(&p, 0, sizeof(p));
  int st;
  for (int t = 0; t < 2; ++t) {
    LinearTier &tr = p.tier[t];
    tr.cols = (int)tiers_cols[t];
    tr.col_offset = (int)tiers_off[t];
    tr.cta_begin = t == 0 ? 0 : hc;
    tr.cta_count = ctas[t];
    tr.ksplit = 1;
    if (tr.cols > 0 && tr.cta_count > 0 &&
        (st = tile_map_2d(&tr.wmap, tiers_w[t], a->dtype, a->K, tiers_cols[t], tiers_ld[t], kBoxCols,
                          linear_wide_k_rows(), 128)))
      return st;
  }
  const void *x = static_cast<const uint16_t *>(a->x) + t0 * a->ldx;
  if ((st = tile_map_2d(&p.xmap, x, a->dtype, nt, a->K, a->ldx, kBoxCols, kMmaMaxTok, 128))) return st;
  p.y = static_cast<uint16_t *>(a->y) + t0 * a->ldy;
  p.ldy = a->ldy;
  p.ntok = (int)nt;
  p.K = (int)a->K;
  p.status = dev->status;
  p.pdl = pdl_enabled() ? 1 : 0;
  p.tok_slices = pair ? (int)((nt + kMmaMaxTok - 1) / kMmaMaxTok) : 0;
  const size_t smem = linear_wide_smem_bytes(pair);
  if ((int)smem > dev->max_smem_optin) return fail(DAK_ERR_UNSUPPORTED, "wide linear: shared memory plan too large");
  if (trace_plans())
    fprintf(stderr, "[dak plan] wide%s ntok=%lld K=%lld host_cols=%lld dev_cols=%lld | host ctas=%d | dev ctas=%d"
            " x %d rows\n", pair ? " paired" : "", (long long)nt, (long long)a->K, (long long)a->host_cols,
            (long long)a->dev_cols, hc, dc, std::max(1, p.tok_slices));
  const cudaError_t e = launch_linear_wide(p, a->dtype, hc + dc, smem, stream, pair);
  return e == cudaSuccess ? DAK_OK : cuda_status(e, "wide linear kernel launch");
}

// Paired wide plan for an HBM-only chunk of 257..512 tokens: the CTAs per
// 256-token row, or 0 when token rows of the tcgen05 kernel move fewer
// operand bytes.  Both plans are costed as the token-row planner costs its
// own: the bytes the busiest CTA brings into shared memory per K row.  A
// paired unit (two 128-feature tiles, 256 tokens) brings 512 bytes of weights
// and 512 of activations; a 128-feature tile of w tokens, 256 and 2w.  Both
// kernels keep one CTA per SM.
int paired_wide_groups(const dak_linear_args *a, const DeviceInfo *dev, int64_t nt) {
  if (a->dev_cols <= 0 || a->host_cols > 0 || nt <= kMmaMaxTok || nt > 2 * kMmaMaxTok) return 0;
  if ((int)linear_wide_smem_bytes(true) > dev->max_smem_optin) return 0;
  const int cap = dev->num_sms;
  const int boxes = (int)((a->dev_cols + kBoxCols - 1) / kBoxCols);
  auto busiest = [&](int units, int rows, long unit_bytes, int *groups_out) -> long {
    int groups = std::min(units, cap / rows);
    if (groups <= 0) return -1;
    const int per = (units + groups - 1) / groups;
    if (groups_out) *groups_out = (units + per - 1) / per;
    return (long)per * unit_bytes;
  };
  int groups = 0;
  const long pair_cost = busiest((boxes + 3) / 4, 2, 1024, &groups);
  if (pair_cost < 0) return 0;
  long best_rows = -1;
  for (int w = kMmaMaxTok; w >= 64; w /= 2) {
    const long c = busiest((boxes + 1) / 2, (int)((nt + w - 1) / w), 256 + 2 * w, nullptr);
    if (c >= 0 && (best_rows < 0 || c < best_rows)) best_rows = c;
  }
  return (best_rows < 0 || 20 * pair_cost < 19 * best_rows) ? groups : 0;
}

int run_linear(const dak_linear_args *a, cudaStream_t stream, const ArParams *ar = nullptr, bool glu = false) {
  if (!a) return fail(DAK_ERR_INVALID_ARG, "args is null");
  if (a->dtype != DAK_DTYPE_F16 && a->dtype != DAK_DTYPE_BF16)
    return fail(DAK_ERR_UNSUPPORTED, "linear supports float16 and bfloat16 only");
  if (a->ntok <= 0 || a->K <= 0) return fail(DAK_ERR_INVALID_ARG, "ntok and K must be positive");
  if (a->host_cols < 0 || a->dev_cols < 0 || a->host_cols + a->dev_cols <= 0)
    return fail(DAK_ERR_INVALID_ARG, "no output features");
  if (a->K > (1ll << 31) || a->host_cols > (1ll << 31) || a->dev_cols > (1ll << 31))
    return fail(DAK_ERR_INVALID_ARG, "dimension too large");
  if (!a->x || !a->y) return fail(DAK_ERR_INVALID_ARG, "x and y are required");
  int st;
  if ((st = check_ptr16(a->x, "x"))) return st;
  if (a->ldx < a->K || (a->ldx % 8) != 0)
    return fail(DAK_ERR_ALIGNMENT, "x row stride must be >= K and a multiple of 8 elements");
  if (a->ldy <= 0) return fail(DAK_ERR_INVALID_ARG, "y row stride must be positive");
  const int64_t tiers_cols[2] = {a->host_cols, a->dev_cols};
  const void *tiers_w[2] = {a->w_host, a->w_dev};
  const int64_t tiers_ld[2] = {a->ld_host, a->ld_dev};
  const int64_t tiers_off[2] = {a->host_col_offset, a->dev_col_offset};
  for (int t = 0; t < 2; ++t) {
    if (tiers_cols[t] == 0) continue;
    const char *nm = t == 0 ? "host weight" : "device weight";
    if (!tiers_w[t]) return fail(DAK_ERR_INVALID_ARG, "%s is null", nm);
    if ((st = check_ptr16(tiers_w[t], nm))) return st;
    if (tiers_ld[t] < tiers_cols[t] || (tiers_ld[t] % 8) != 0)
      return fail(DAK_ERR_ALIGNMENT, "%s row stride must be >= its columns and a multiple of 8", nm);
    if (glu && (tiers_cols[t] % 32 != 0 || tiers_off[t] % 32 != 0))
      return fail(DAK_ERR_INVALID_ARG, "gated linear: %s columns and offset must be multiples of 32", nm);
    // A gated linear writes half as many y columns as the weight has features.
    if (tiers_off[t] < 0 || (tiers_off[t] + tiers_cols[t]) / (glu ? 2 : 1) > a->ldy)
      return fail(DAK_ERR_INVALID_ARG, "%s columns fall outside y", nm);
  }

  DeviceInfo *dev;
  if ((st = device_info(&dev))) return st;

  int path = a->path;
  if (path == DAK_PATH_AUTO) path = a->ntok <= kCoreAutoMaxTok ? DAK_PATH_CUDA_CORE : DAK_PATH_TCGEN05;
  if (ar || glu) {
    // The fused all-reduce and the gated epilogue live in the tcgen05 kernel,
    // which serves any token count.
    if (a->path == DAK_PATH_CUDA_CORE)
      return fail(DAK_ERR_UNSUPPORTED, "the %s runs on the tcgen05 path", ar ? "fused all-reduce" : "gated linear");
    path = DAK_PATH_TCGEN05;
  }
  if (path == DAK_PATH_CUDA_CORE && a->ntok > kCoreMaxTok)
    return fail(DAK_ERR_INVALID_ARG, "CUDA-core path serves at most %d tokens", kCoreMaxTok);
  const bool mma = path == DAK_PATH_TCGEN05;
  const int bn = mma ? kMmaBM : kCoreBN;
  const int bk = mma ? kMmaBK : kCoreBK;
  const int max_ks = mma ? kMmaMaxKsplitHost : kCoreMaxKsplit;
  const int nkb = (int)((a->K + bk - 1) / bk);

  // Token chunks: the tcgen05 kernel serves up to 256 tokens per grid row; the
  // wide kernel up to 512 for a layer with host-resident rows, so that those
  // rows cross the host link once per 512 tokens instead of once per 256.  An
  // HBM-only layer also takes up to 512 tokens per launch, as grid rows of 64
  // to 256 tokens (token slices, planned below), so that each weight tile is
  // brought into shared memory once per 512 tokens at about the same time by
  // every row, not once per 256-token launch.
  const bool wide = mma && !ar && !glu && a->host_cols > 0 && a->ntok > kMmaMaxTok;
  const bool sliced = mma && !ar && !glu && a->host_cols == 0 && a->ntok > kMmaMaxTok && a->host_ctas <= 0 &&
                      a->dev_ctas <= 0;
  const int64_t chunk = (wide || sliced) ? 2 * kMmaMaxTok : mma ? kMmaMaxTok : kCoreMaxTok;
  for (int64_t t0 = 0; t0 < a->ntok; t0 += chunk) {
    const int64_t nt = std::min(chunk, a->ntok - t0);
    if (wide && nt > kMmaMaxTok) {
      if ((st = run_linear_wide_chunk(a, dev, t0, nt, stream))) return st;
      continue;
    }
    if (sliced && nt > kMmaMaxTok) {
      const int pg = paired_wide_groups(a, dev, nt);
      if (pg > 0) {
        if ((st = run_linear_wide_chunk(a, dev, t0, nt, stream, pg))) return st;
        continue;
      }
    }
    int tmpl = 1;
    if (mma) {
      tmpl = 16;
      while (tmpl < nt && tmpl < kMmaMaxTok) tmpl *= 2;  // a chunk above 256 tokens must take token rows
    } else {
      while (tmpl < nt) tmpl *= 2;
    }

    // ---- plan the two tiers
    const int tiles_h = (int)((a->host_cols + bn - 1) / bn);
    const int tiles_d = (int)((a->dev_cols + bn - 1) / bn);
    // Resident CTAs of one wave for a cluster size (cudaOccupancyMaxActiveClusters).
    auto capacity = [&](int cl) -> int {
      const size_t sm = mma ? linear_mma_smem_bytes(tmpl, cl - 1) : linear_core_smem_bytes(tmpl, cl - 1);
      if (sm == 0 || (int)sm > dev->max_smem_optin) return 0;
      return max_resident_ctas(mma, tmpl, a->dtype, cl, sm, dev->num_sms);
    };
    TierPlan ph, pd;
    int cluster = 1;
    int tok_slices = 1;  // grid rows of tmpl tokens each (tcgen05, HBM-only layers)
    // Largest split factor whose split-K receive buffer still fits with at
    // least two pipeline stages.
    int ks_cap = 1;
    for (int ks = 2; ks <= max_ks; ks *= 2) {
      const size_t sm = mma ? linear_mma_smem_bytes(tmpl, ks - 1) : linear_core_smem_bytes(tmpl, ks - 1);
      if (sm == 0 || (int)sm > dev->max_smem_optin) break;
      ks_cap = ks;
    }
    if (a->host_ctas > 0 || a->dev_ctas > 0) {
      ph = user_plan(a->host_ctas, std::max(1, a->host_ksplit), tiles_h, nkb, ks_cap);
      pd = user_plan(a->dev_ctas, std::max(1, a->dev_ksplit), tiles_d, nkb, ks_cap);
      if (tiles_h > 0 && ph.ctas == 0) ph = user_plan(1, 1, tiles_h, nkb, ks_cap);
      if (tiles_d > 0 && pd.ctas == 0) pd = user_plan(1, 1, tiles_d, nkb, ks_cap);
      cluster = std::max(ph.ksplit, pd.ksplit);
      if (cluster % ph.ksplit != 0 || cluster % pd.ksplit != 0) {
        // Incompatible split factors share one launch shape: fall back to no split.
        ph.ksplit = pd.ksplit = 1;
        cluster = 1;
      }
    } else {
      const int hb = tiles_h > 0 ? std::min(kAutoHostCtas, dev->num_sms / 4) : 0;
      ph = auto_plan(hb, tiles_h, nkb, ks_cap);
      cluster = ph.ksplit;
      if (tiles_d > 0) {
        // Device-tier plan, from launch-plan sweeps of these kernels on B200
        // (the Llama-3-8B layers and one TP8 rank's Llama-3-70B layers, chained
        // in CUDA graphs): give each group whole tiles (full-width stages
        // stream fastest) and split K only as far as needed to bring about
        // 1 MB of weight per CTA (at least 96 CTAs), because every split adds
        // a DSMEM reduction per tile.  A split never leaves a CTA fewer than
        // kMinSplitRows K rows, and it stops at a balanced plan within 3/4 of
        // the target rather than take one that gives some groups two tiles
        // and others one.  With at least 3/4 of a wave of tiles, no split:
        // tiles are spread evenly over the resident CTAs.
        long best_cost = -1;
        TierPlan best;
        int best_cluster = cluster;
        const int boxes_d = (int)((a->dev_cols + kBoxCols - 1) / kBoxCols);
        const int bpt = bn / kBoxCols;  // boxes per full tile
        const int tiles_full = (boxes_d + bpt - 1) / bpt;
        const double w_bytes = 2.0 * (double)a->dev_cols * (double)a->K;
        const int cl1 = std::max(1, ph.ksplit);
        const int cap1 = capacity(cl1) - (ph.ctas + cl1 - 1) / cl1 * cl1;
        if (cap1 > 0 && ph.ksplit == 1 && 4 * tiles_full >= 3 * cap1) {
          const int per = (tiles_full + cap1 - 1) / cap1;  // tiles per group
          best.ksplit = 1;
          best.ctas = (tiles_full + per - 1) / per;
          best_cluster = 1;
          best_cost = 0;
        } else {
          const int target = std::max(96, (int)(w_bytes / 1.0e6));
          const int ks_rows = std::max(1, (int)(a->K / kMinSplitRows));
          for (int ks = 1; ks <= ks_cap && ks <= std::max(1, nkb) && (ks == 1 || ks <= ks_rows); ks *= 2) {
            const int cl = std::max(ks, ph.ksplit);
            const int cap = capacity(cl) - (ph.ctas + cl - 1) / cl * cl;
            const int groups = std::min(cap / ks, tiles_full);
            if (groups <= 0) continue;
            if (best_cost >= 0 && groups < tiles_full && 4 * best.ctas >= 3 * target) break;
            best.ksplit = ks;
            best.ctas = groups * ks;
            best_cluster = cl;
            best_cost = 0;
            if (best.ctas >= target || groups < tiles_full) break;
          }
        }
        if (best_cost < 0) {  // no occupancy answer: one tile per CTA, no split
          best = auto_plan(std::max(1, dev->num_sms - ph.ctas), tiles_d, nkb, 1);
          best_cluster = ph.ksplit;
        }
        pd = best;
        cluster = best_cluster;
      }
      // Token slices.  Above 64 tokens a CTA's time follows the operand
      // bytes it moves into shared memory: per K row, a tile of 128 features
      // brings 256 bytes of weights plus 2 bytes per token of activations.
      // And split-K's receive buffer no longer fits beside the stages, so a
      // narrow HBM-only layer would leave most SMs idle (4096 output
      // features: 32 CTAs).  Grid rows of 64 or 128 tokens give a layer more
      // CTAs with smaller stages; the rows read the same weight tiles at about
      // the same time, mostly from L2.  The plan with the fewest bytes for its
      // busiest CTA wins (by at least 5%); on the Llama-3-8B layers at 256
      // tokens this model orders the 1-, 2- and 4-row plans as their measured
      // times do.
      // A chunk of more tokens than one row holds (257..512) always takes
      // rows: the row width with the fewest operand bytes for its busiest
      // CTA, 256 included.
      const bool must_slice = nt > tmpl;
      if (mma && !ar && tiles_h == 0 && pd.ctas > 0 && pd.ksplit == 1 && tmpl >= 128) {
        const int boxes = (int)((a->dev_cols + kBoxCols - 1) / kBoxCols);
        const int bpt = bn / kBoxCols;
        auto busiest_cost = [&](int groups, int w) -> long {
          const int tiles = ((boxes + groups - 1) / groups + bpt - 1) / bpt;  // the busiest group's tiles
          return (long)tiles * (256 + 2 * w);
        };
        long best_cost = must_slice ? -1 : busiest_cost(pd.ctas, tmpl);
        int best_w = 0, best_groups = 0, best_rows = 1;
        const int tiles_all = (boxes + bpt - 1) / bpt;
        for (int sl = must_slice ? 1 : 2; sl <= 4 && tmpl / sl >= 64; sl *= 2) {
          const int w = tmpl / sl;
          const int rows = (int)((nt + w - 1) / w);
          const size_t sm = linear_mma_smem_bytes(w, 0);
          if (sm == 0 || (int)sm > dev->max_smem_optin) continue;
          const int cap = max_resident_ctas(true, w, a->dtype, 1, sm, dev->num_sms);
          int groups = std::min(tiles_all, cap / rows);
          if (groups <= 0) continue;
          const int per = (tiles_all + groups - 1) / groups;
          groups = (tiles_all + per - 1) / per;  // the fewest groups with that many tiles each
          const long cost = busiest_cost(groups, w);
          if (best_cost < 0 || 20 * cost < 19 * best_cost) {
            best_cost = cost;
            best_w = w;
            best_groups = groups;
            best_rows = rows;
          }
        }
        if (best_w > 0) {
          tmpl = best_w;
          pd.ctas = best_groups;
          tok_slices = best_rows;
        }
      }
    }
    if ((int64_t)std::max(1, tok_slices) * tmpl < nt)
      return fail(DAK_ERR_UNSUPPORTED, "linear: no token-row plan covers %lld tokens", (long long)nt);
    const int span_h = (ph.ctas + cluster - 1) / cluster * cluster;
    const int span_d = (pd.ctas + cluster - 1) / cluster * cluster;
    const int grid = span_h + span_d;
    if (trace_plans())
      fprintf(stderr,
              "[dak plan] %s ntok=%lld K=%lld host_cols=%lld dev_cols=%lld | host ctas=%d ks=%d | dev ctas=%d ks=%d"
              " | cluster=%d grid=%d x %d rows of %d tokens | cap=%d\n",
              mma ? "tcgen05" : "core", (long long)nt, (long long)a->K, (long long)a->host_cols,
              (long long)a->dev_cols, ph.ctas, ph.ksplit, pd.ctas, pd.ksplit, cluster, grid, tok_slices, tmpl,
              capacity(cluster));

    LinearParams p;
    std::memset(&p, 0, sizeof(p));
    const int64_t plan_ctas[2] = {ph.ctas, pd.ctas};
    const int plan_ks[2] = {ph.ksplit, pd.ksplit};
    const int begins[2] = {0, span_h};
    for (int t = 0; t < 2; ++t) {
      LinearTier &tr = p.tier[t];
      tr.cols = (int)tiers_cols[t];
      tr.col_offset = (int)tiers_off[t];
      tr.cta_begin = begins[t];
      tr.cta_count = (int)plan_ctas[t];
      tr.ksplit = plan_ks[t];
      if (tr.cols > 0 && tr.cta_count > 0) {
        st = tile_map_2d(&tr.wmap, tiers_w[t], a->dtype, a->K, tiers_cols[t], tiers_ld[t], kBoxCols,
                         bk, 128);
        if (st) return st;
      }
    }
    const void *x = static_cast<const uint16_t *>(a->x) + t0 * a->ldx;
    if (mma)
      st = tile_map_2d(&p.xmap, x, a->dtype, nt, a->K, a->ldx, kBoxCols, tmpl, 128);  // two 64-wide boxes per stage
    else
      st = tile_map_2d(&p.xmap, x, a->dtype, nt, a->K, a->ldx, kCoreBK, tmpl, 0);
    if (st) return st;
    p.y = static_cast<uint16_t *>(a->y) + t0 * a->ldy;
    p.ldy = a->ldy;
    p.ntok = (int)nt;
    p.K = (int)a->K;
    p.status = dev->status;
    p.red_slots = cluster - 1;
    p.pdl = pdl_enabled() ? 1 : 0;
    p.tok_slices = tok_slices;
    p.glu = glu ? 1 : 0;
    if (ar) {
      if (grid > kArMaxCtas) return fail(DAK_ERR_UNSUPPORTED, "fused all-reduce: grid of %d CTAs", grid);
      if (ar->slot_elems < nt * a->ldy)
        return fail(DAK_ERR_INVALID_ARG, "fused all-reduce: slot_elems %lld below %lld x ldy",
                    (long long)ar->slot_elems, (long long)nt);
      p.ar_on = 1;
      p.ar = *ar;
    }

    size_t smem;
    cudaError_t e;
    if (mma) {
      p.stages = linear_mma_stages(tmpl, cluster);
      smem = linear_mma_smem_bytes(tmpl, cluster - 1);
      if (smem == 0 || (int)smem > dev->max_smem_optin)
        return fail(DAK_ERR_UNSUPPORTED, "tcgen05 linear: no shared-memory plan for %d tokens, split %d",
                    tmpl, cluster);
      e = launch_linear_mma(p, tmpl, a->dtype, grid, cluster, smem, stream);
    } else {
      p.stages = linear_core_stages(tmpl, cluster - 1);
      smem = linear_core_smem_bytes(tmpl, cluster - 1);
      if (smem == 0 || (int)smem > dev->max_smem_optin)
        return fail(DAK_ERR_UNSUPPORTED, "linear: shared memory plan exceeds the device limit");
      e = launch_linear_core(p, tmpl, a->dtype, grid, cluster, smem, stream);
    }
    if (e != cudaSuccess) return cuda_status(e, "linear kernel launch");
  }
  return DAK_OK;
}

// Shared by the reference-shaped entry points: A descriptors -> tiers.
int gemv_from_descs(const void *a_h, const void *a_d, const void *b, const void *c, int h_M,
                    int d_M, int N, int K, int num_copy_blocks, int num_copy_host_blocks,
                    int h_spr, int d_spr, cudaStream_t stream) {
  if (h_M < 0 || d_M < 0 || N <= 0 || K <= 0)
    return fail(DAK_ERR_INVALID_ARG, "M, N, K must be positive");
  MatView ah{}, ad{}, bv{}, cv{};
  int st;
  if (h_M > 0 && (st = desc_to_matrix(a_h, "A (host rows)", &ah))) return st;
  if (d_M > 0 && (st = desc_to_matrix(a_d, "A (device rows)", &ad))) return st;
  if ((st = desc_to_matrix(b, "B", &bv))) return st;
  if ((st = desc_to_matrix(c, "C", &cv))) return st;
  const int dtype = bv.dtype;
  if (h_M > 0 && (ah.cols != h_M || ah.rows != K || ah.dtype != dtype))
    return fail(DAK_ERR_INVALID_ARG, "A (host rows) is [%lld x %lld], expected [K=%d x %d]",
                (long long)ah.rows, (long long)ah.cols, K, h_M);
  if (d_M > 0 && (ad.cols != d_M || ad.rows != K || ad.dtype != dtype))
    return fail(DAK_ERR_INVALID_ARG, "A (device rows) is [%lld x %lld], expected [K=%d x %d]",
                (long long)ad.rows, (long long)ad.cols, K, d_M);
  if (bv.cols != K || bv.rows != N)
    return fail(DAK_ERR_INVALID_ARG, "B is [%lld x %lld], expected [N=%d x K=%d]", (long long)bv.rows,
                (long long)bv.cols, N, K);
  if (cv.cols != (int64_t)h_M + d_M || cv.rows != N || cv.dtype != dtype)
    return fail(DAK_ERR_INVALID_ARG, "C is [%lld x %lld], expected [N=%d x M=%d]", (long long)cv.rows,
                (long long)cv.cols, N, h_M + d_M);
  dak_linear_args a;
  std::memset(&a, 0, sizeof(a));
  a.w_host = ah.base;
  a.host_cols = h_M;
  a.ld_host = ah.ld;
  a.host_col_offset = 0;
  a.w_dev = ad.base;
  a.dev_cols = d_M;
  a.ld_dev = ad.ld;
  a.dev_col_offset = h_M;
  a.x = bv.base;
  a.ldx = bv.ld;
  a.y = const_cast<void *>(cv.base);
  a.ldy = cv.ld;
  a.ntok = N;
  a.K = K;
  a.dtype = dtype;
  if (num_copy_blocks > 0) {
    const int hb = std::max(0, std::min(num_copy_host_blocks, num_copy_blocks));
    a.host_ctas = h_M > 0 ? std::max(1, hb) : 0;
    a.dev_ctas = d_M > 0 ? std::max(1, num_copy_blocks - hb) : 0;
    a.host_ksplit = std::max(1, h_spr);
    a.dev_ksplit = std::max(1, d_spr);
  }
  // The single-tier entry points (`gemv`, linearLayer.py:72-80 with the weight
  // moved to "cpu") pass a pinned host weight as their only tier.  For batches
  // above one tcgen05 launch, serve it as the host tier, so that it takes the
  // kernel that streams host rows once for up to 512 tokens.
  if (h_M == 0 && d_M > 0 && N > kMmaMaxTok) {
    cudaPointerAttributes attr;
    if (cudaPointerGetAttributes(&attr, ad.base) == cudaSuccess && attr.type == cudaMemoryTypeHost) {
      std::swap(a.w_host, a.w_dev);
      std::swap(a.host_cols, a.dev_cols);
      std::swap(a.ld_host, a.ld_dev);
      a.host_col_offset = 0;
      a.dev_col_offset = 0;
      std::swap(a.host_ctas, a.dev_ctas);
      std::swap(a.host_ksplit, a.dev_ksplit);
    } else {
      cudaGetLastError();
    }
  }
  a.path = DAK_PATH_AUTO;
  return run_linear(&a, stream);
}
}  // namespace

// ------------------------------------------------------------ utility kernels
namespace {
__global__ void flush_l2_kernel(const float *buf, size_t n, float *sink) {
  float acc = 0.f;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
       i += (size_t)blockDim.x * gridDim.x)
    acc += __ldcg(buf + i);
  if (acc == 1234.5678f) *sink += acc;  // keeps the loads alive
}

// Streams [src, src+bytes) through shared memory with `stages` bulk copies of
// `chunk` bytes in flight per CTA; returns an XOR checksum of the data.
__global__ void probe_read_kernel(const uint8_t *src, size_t bytes, int stages, int chunk,
                                  uint32_t *sink, int *status) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ uint64_t bars[16];
  __shared__ int abort_flag;
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t *smem = smem_raw + (((raw + 127u) & ~127u) - raw);
  const size_t per = (bytes / gridDim.x) & ~(size_t)15;
  const uint8_t *beg = src + per * blockIdx.x;
  const size_t len = blockIdx.x + 1 == gridDim.x ? (bytes - per * blockIdx.x) & ~(size_t)15 : per;
  const size_t nch = (len + chunk - 1) / chunk;
  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) mbar_init(smem_u32(&bars[s]), 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  const WaitCtx wc{&abort_flag, status};
  uint32_t x = 0;
  if (threadIdx.x == 0) {
    const uint64_t pol = l2_policy_evict_first();
    size_t issued = 0;
    for (; issued < nch && issued < (size_t)stages; ++issued) {
      const size_t off = issued * chunk;
      const uint32_t n = (uint32_t)std::min<size_t>(chunk, len - off);
      const uint32_t b = smem_u32(&bars[issued % stages]);
      mbar_arrive_expect_tx(b, n);
      bulk_load(smem_u32(smem + (issued % stages) * chunk), beg + off, n, b, pol);
    }
    for (size_t i = 0; i < nch; ++i) {
      const int s = (int)(i % stages);
      const uint32_t par = (uint32_t)((i / stages) & 1);
      if (!mbar_wait<false>(smem_u32(&bars[s]), par, wc)) break;
      x ^= *reinterpret_cast<const uint32_t *>(smem + s * chunk);
      if (issued < nch) {
        const size_t off = issued * chunk;
        const uint32_t n = (uint32_t)std::min<size_t>(chunk, len - off);
        mbar_arrive_expect_tx(smem_u32(&bars[s]), n);
        bulk_load(smem_u32(smem + s * chunk), beg + off, n, smem_u32(&bars[s]), pol);
        ++issued;
      }
    }
    atomicXor(sink, x);
  }
}
// A wait that nothing completes: gives up after timeout_ns, leaving
// DAK_ERR_TIMEOUT in the status word (the path every kernel takes when a copy
// or a peer never arrives).
__global__ void selftest_wait_kernel(int *status, unsigned long long timeout_ns) {
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(smem_u32(&bar), 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  const WaitCtx wc{&abort_flag, status};
  mbar_wait<false>(smem_u32(&bar), 0, wc, timeout_ns);
}
}  // namespace

}  // namespace dak

// =================================================================== C ABI
using namespace dak;

extern "C" {

const char *dak_strerror(int status) {
  switch (status) {
    case DAK_OK: return "success";
    case DAK_ERR_INVALID_ARG: return "invalid argument";
    case DAK_ERR_UNSUPPORTED: return "unsupported";
    case DAK_ERR_CUDA: return "CUDA runtime error";
    case DAK_ERR_DRIVER: return "CUDA driver error";
    case DAK_ERR_TIMEOUT: return "device wait timed out";
    case DAK_ERR_ALIGNMENT: return "misaligned pointer or stride";
    case DAK_ERR_NO_DEVICE: return "no CUDA device";
    default: return "unknown status";
  }
}

const char *dak_last_error_message(void) { return t_last_error; }

int dak_get_constants(dak_constants *out) {
  if (!out) return fail(DAK_ERR_INVALID_ARG, "out is null");
  int num_sms = 148;  // B200; replaced by the live count when a device is visible
  int dev = 0;
  if (cudaGetDevice(&dev) == cudaSuccess) {
    int v = 0;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess && v > 0)
      num_sms = v;
  } else {
    cudaGetLastError();
  }
  out->num_sms = num_sms;
  out->max_copy_sms = num_sms;
  out->buffer_slots = kCoreStages;
  out->tile_n = kCoreMaxTok;
  out->tile_m = 64;
  out->tile_k = kCoreBK;
  out->mma_tile_m = kMmaBM;
  out->mma_max_tokens = kMmaMaxTok;
  out->abi_version = 1;
  return DAK_OK;
}

int dak_print_device_name(int device_id) {
  cudaDeviceProp prop;
  cudaError_t e = cudaGetDeviceProperties(&prop, device_id);
  if (e != cudaSuccess) return cuda_status(e, "cudaGetDeviceProperties");
  printf("Running on device %d: %s\n", device_id, prop.name);
  fflush(stdout);
  return DAK_OK;
}

size_t dak_set_smem_size(size_t smem_size, int opcode) {
  if (opcode < DAK_OP_GEMV || opcode > DAK_OP_GEMV_HORIZONTAL_MULTICAST_PREFILL) {
    fail(DAK_ERR_INVALID_ARG, "Unsupported opcode: %d", opcode);
    return 0;
  }
  DeviceInfo *dev;
  if (device_info(&dev) == DAK_OK && smem_size > (size_t)dev->max_smem_optin) {
    fail(DAK_ERR_INVALID_ARG, "shared memory request %zu exceeds the device limit %d", smem_size,
         dev->max_smem_optin);
    return 0;
  }
  return smem_size;
}

int dak_build_tma_desc(void *desc_out, const void *base, int dtype, int rank,
                       const int64_t *shape, const int64_t *strides_bytes,
                       const int64_t *box_dim, const int64_t *elem_strides, int swizzle_bytes) {
  if (!desc_out) return fail(DAK_ERR_INVALID_ARG, "desc_out is null");
  if (!base) return fail(DAK_ERR_INVALID_ARG, "base must have storage");
  if (rank < 1 || rank > 5)
    return fail(DAK_ERR_INVALID_ARG, "tensorRank=%d not supported here (adjust if needed)", rank);
  const int es = elem_size(dtype);
  if (es == 0) return fail(DAK_ERR_UNSUPPORTED, "Unsupported tensor dtype for TMA: %d", dtype);
  if (swizzle_bytes != 0 && swizzle_bytes != 32 && swizzle_bytes != 64 && swizzle_bytes != 128)
    return fail(DAK_ERR_INVALID_ARG, "Unsupported swizzle_bytes=%d (expected 0/32/64/128)", swizzle_bytes);
  if (!shape || !box_dim || !elem_strides || (rank > 1 && !strides_bytes))
    return fail(DAK_ERR_INVALID_ARG, "shape/strides/box arrays are required");
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0)
    return fail(DAK_ERR_ALIGNMENT, "base address must be 16-byte aligned");
  DescBlob d;
  std::memset(&d, 0, sizeof(d));
  d.magic = kDescMagic;
  d.version = 1;
  d.dtype = (uint8_t)dtype;
  d.rank = (uint8_t)rank;
  d.base = reinterpret_cast<uint64_t>(base);
  for (int i = 0; i < rank; ++i) {
    if (shape[i] <= 0) return fail(DAK_ERR_INVALID_ARG, "shape[%d] must be > 0", i);
    if (box_dim[i] <= 0) return fail(DAK_ERR_INVALID_ARG, "box_dim[%d] must be > 0", i);
    if (box_dim[i] > 256) return fail(DAK_ERR_INVALID_ARG, "box_dim[%d] must be <= 256", i);
    if (elem_strides[i] <= 0 || elem_strides[i] > 8)
      return fail(DAK_ERR_INVALID_ARG, "elem_strides[%d] must be in [1, 8]", i);
    d.shape[i] = (uint64_t)shape[i];
    d.box[i] = (uint16_t)box_dim[i];
    d.elem_strides[i] = (uint8_t)elem_strides[i];
    if (i < rank - 1) {
      if (strides_bytes[i] <= 0) return fail(DAK_ERR_INVALID_ARG, "strides_bytes[%d] must be > 0", i);
      if (strides_bytes[i] % 16 != 0)
        return fail(DAK_ERR_ALIGNMENT, "strides_bytes[%d] must be a multiple of 16", i);
      d.strides[i] = (uint64_t)strides_bytes[i];
    }
  }
  const int64_t inner_bytes = box_dim[0] * es;
  if (inner_bytes % 16 != 0)
    return fail(DAK_ERR_INVALID_ARG, "inner box dimension must span a multiple of 16 bytes");
  if (swizzle_bytes != 0 && inner_bytes > swizzle_bytes)
    return fail(DAK_ERR_INVALID_ARG, "inner box dimension exceeds the %d-byte swizzle span", swizzle_bytes);
  d.swizzle = (uint8_t)(swizzle_bytes == 0 ? 0 : swizzle_bytes == 32 ? 1 : swizzle_bytes == 64 ? 2 : 3);
  std::memcpy(desc_out, &d, sizeof(d));
  return DAK_OK;
}

int dak_tensormap_replace_address(void *desc, const void *new_base) {
  if (!desc || !new_base) return fail(DAK_ERR_INVALID_ARG, "descriptor and address are required");
  DescBlob d;
  std::memcpy(&d, desc, sizeof(d));
  if (d.magic != kDescMagic) return fail(DAK_ERR_INVALID_ARG, "not a DAK descriptor");
  if ((reinterpret_cast<uintptr_t>(new_base) & 15u) != 0)
    return fail(DAK_ERR_ALIGNMENT, "new address must be 16-byte aligned");
  d.base = reinterpret_cast<uint64_t>(new_base);
  std::memcpy(desc, &d, sizeof(d));
  return DAK_OK;
}

int dak_linear_split(const dak_linear_args *args, void *stream) {
  return run_linear(args, static_cast<cudaStream_t>(stream));
}

int dak_linear_split_glu(const dak_linear_args *args, void *stream) {
  return run_linear(args, static_cast<cudaStream_t>(stream), nullptr, true);
}

int dak_linear_split_allreduce(const dak_linear_args *args, const dak_allreduce_args *ar, void *stream) {
  if (!ar) return fail(DAK_ERR_INVALID_ARG, "all-reduce args are null");
  if (ar->world < 1 || ar->world > kArMaxRanks || ar->rank < 0 || ar->rank >= ar->world)
    return fail(DAK_ERR_INVALID_ARG, "world must be 1..%d and rank in [0, world)", kArMaxRanks);
  if (!ar->epoch || !ar->done || ar->slot_elems <= 0 || ar->timeout_us <= 0)
    return fail(DAK_ERR_INVALID_ARG, "epoch, done, slot_elems and timeout_us are required");
  ArParams p;
  std::memset(&p, 0, sizeof(p));
  const bool mc = ar->mc_f32 != nullptr;
  if (mc != (ar->own_f32 != nullptr)) return fail(DAK_ERR_INVALID_ARG, "own_f32 and mc_f32 come together");
  if (mc && ((reinterpret_cast<uintptr_t>(ar->own_f32) & 15u) || (reinterpret_cast<uintptr_t>(ar->mc_f32) & 15u)))
    return fail(DAK_ERR_ALIGNMENT, "own_f32 and mc_f32 must be 16-byte aligned");
  for (int r = 0; r < ar->world; ++r) {
    if ((!mc && !ar->buffers[r]) || !ar->flags[r]) return fail(DAK_ERR_INVALID_ARG, "rank %d buffer or flags missing", r);
    if ((reinterpret_cast<uintptr_t>(ar->buffers[r]) & 15u) || (reinterpret_cast<uintptr_t>(ar->flags[r]) & 3u))
      return fail(DAK_ERR_ALIGNMENT, "rank %d buffer must be 16-byte aligned, flags 4-byte aligned", r);
    p.buf[r] = static_cast<uint16_t *>(ar->buffers[r]);
    p.flags[r] = ar->flags[r];
  }
  p.own = ar->own_f32;
  p.mc = ar->mc_f32;
  if (ar->publish_only && !mc) return fail(DAK_ERR_INVALID_ARG, "publish_only needs the multicast buffers");
  p.publish_only = ar->publish_only ? 1 : 0;
  p.slot_elems = ar->slot_elems;
  p.epoch = ar->epoch;
  p.done = ar->done;
  p.world = ar->world;
  p.rank = ar->rank;
  p.timeout_ns = ar->timeout_us * 1000;
  return run_linear(args, static_cast<cudaStream_t>(stream), &p);
}

int dak_gemv(const void *a_desc, const void *b_desc, const void *c_desc, int M, int N, int K,
             int num_copy_blocks, int smem_size, int sms_per_row, void *stream) {
  (void)smem_size;
  return gemv_from_descs(nullptr, a_desc, b_desc, c_desc, 0, M, N, K, num_copy_blocks, 0, 1,
                         sms_per_row, static_cast<cudaStream_t>(stream));
}

int dak_gemv_horizontal(const void *a_desc_h, const void *a_desc_d, const void *b_desc,
                        const void *c_desc, int h_M, int d_M, int N, int K, int num_copy_blocks,
                        int num_copy_host_blocks, int smem_size, int h_sms_per_row,
                        int d_sms_per_row, void *stream) {
  (void)smem_size;
  return gemv_from_descs(a_desc_h, a_desc_d, b_desc, c_desc, h_M, d_M, N, K, num_copy_blocks,
                         num_copy_host_blocks, h_sms_per_row, d_sms_per_row,
                         static_cast<cudaStream_t>(stream));
}

int dak_gemv_multicast(const void *a_desc, const void *b_desc, const void *c_desc, int M, int N,
                       int K, int num_copy_blocks, int smem_size, int sms_per_row, void *stream) {
  return dak_gemv(a_desc, b_desc, c_desc, M, N, K, num_copy_blocks, smem_size, sms_per_row, stream);
}

int dak_gemv_multicast_prefill(const void *a_desc, const void *b_desc, const void *c_desc, int M,
                               int N, int K, int num_copy_blocks, int smem_size, int sms_per_row,
                               void *stream) {
  return dak_gemv(a_desc, b_desc, c_desc, M, N, K, num_copy_blocks, smem_size, sms_per_row, stream);
}

int dak_gemv_horizontal_multicast(const void *a_desc_h, const void *a_desc_d, const void *b_desc,
                                  const void *c_desc, int h_M, int d_M, int N, int K,
                                  int num_copy_blocks, int num_copy_host_blocks, int smem_size,
                                  int h_sms_per_row, int d_sms_per_row, void *stream) {
  return dak_gemv_horizontal(a_desc_h, a_desc_d, b_desc, c_desc, h_M, d_M, N, K, num_copy_blocks,
                             num_copy_host_blocks, smem_size, h_sms_per_row, d_sms_per_row, stream);
}

int dak_gemv_horizontal_multicast_prefill(const void *a_desc_h, const void *a_desc_d,
                                          const void *b_desc, const void *c_desc, int h_M,
                                          int d_M, int N, int K, int num_copy_blocks,
                                          int num_copy_host_blocks, int smem_size,
                                          int h_sms_per_row, int d_sms_per_row, void *stream) {
  return dak_gemv_horizontal(a_desc_h, a_desc_d, b_desc, c_desc, h_M, d_M, N, K, num_copy_blocks,
                             num_copy_host_blocks, smem_size, h_sms_per_row, d_sms_per_row, stream);
}

int dak_flush_l2_cache(float *dummy, size_t n, float *sink, void *stream) {
  if (!dummy || !sink) return fail(DAK_ERR_INVALID_ARG, "dummy and sink are required");
  DeviceInfo *dev;
  int st = device_info(&dev);
  if (st) return st;
  flush_l2_kernel<<<dev->num_sms * 4, 256, 0, static_cast<cudaStream_t>(stream)>>>(dummy, n, sink);
  return cuda_status(cudaGetLastError(), "flush_l2_cache launch");
}

int dak_device_status(int clear, int *status_out) {
  DeviceInfo *dev;
  int st = device_info(&dev);
  if (st) return st;
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return cuda_status(e, "cudaDeviceSynchronize");
  int v = 0;
  e = cudaMemcpyFromSymbol(&v, g_dak_status, sizeof(int));
  if (e != cudaSuccess) return cuda_status(e, "read status word");
  if (clear) {
    const int zero = 0;
    e = cudaMemcpyToSymbol(g_dak_status, &zero, sizeof(int));
    if (e != cudaSuccess) return cuda_status(e, "clear status word");
  }
  if (status_out) *status_out = v;
  return DAK_OK;
}

int dak_selftest_wait_timeout(unsigned int timeout_us, void *stream) {
  if (timeout_us == 0 || timeout_us > 10000000u)
    return fail(DAK_ERR_INVALID_ARG, "timeout_us must be in (0, 10 s]");
  DeviceInfo *dev;
  int st = device_info(&dev);
  if (st) return st;
  selftest_wait_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(dev->status,
                                                                        (unsigned long long)timeout_us * 1000ull);
  return cuda_status(cudaGetLastError(), "selftest launch");
}

int dak_probe_stream_read(const void *src, size_t bytes, int ctas, int stages, int chunk_bytes,
                          uint32_t *sink, void *stream) {
  if (!src || !sink || bytes < 16) return fail(DAK_ERR_INVALID_ARG, "src, sink and bytes are required");
  if (ctas <= 0 || stages <= 0 || stages > 16 || chunk_bytes < 16 || chunk_bytes % 16 != 0)
    return fail(DAK_ERR_INVALID_ARG, "need ctas > 0, 1 <= stages <= 16, chunk_bytes a multiple of 16");
  if ((reinterpret_cast<uintptr_t>(src) & 15u) != 0) return fail(DAK_ERR_ALIGNMENT, "src must be 16-byte aligned");
  DeviceInfo *dev;
  int st = device_info(&dev);
  if (st) return st;
  const size_t smem = (size_t)stages * chunk_bytes + 128;
  if ((int)smem > dev->max_smem_optin) return fail(DAK_ERR_INVALID_ARG, "stages x chunk exceeds shared memory");
  cudaError_t e = cudaFuncSetAttribute(probe_read_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return cuda_status(e, "probe attribute");
  probe_read_kernel<<<ctas, 32, smem, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint8_t *>(src), bytes, stages, chunk_bytes, sink, dev->status);
  return cuda_status(cudaGetLastError(), "probe launch");
}

}  // extern "C"
