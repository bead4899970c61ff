// dak_decode_ops.cu - the element-wise steps of a Llama decode layer around the
// offloaded linears and the decode attention: RMSNorm (with the residual add
// fused in), rotary embedding of q and k, and the SiLU-gated product.
//
// The reference runs these as separate torch ops inside its vendored model
// (app/python/llama/vanila_llama.py:227-400, from transformers' Llama); one
// decode layer then costs ~35 tiny launches besides the linears.  Each kernel
// here follows those ops' arithmetic, including the roundings to 16 bit
// between them, so results match transformers to within FP32 reduction order.
#include <algorithm>
#include <cstring>

#include "dak_common.cuh"
#include "dak_host.h"

namespace dak {
namespace {

template <typename T> __device__ __forceinline__ float ld1(const void *p, long long i) {
  return Elem<T>::to_float(reinterpret_cast<const uint16_t *>(p)[i]);
}
template <typename T> __device__ __forceinline__ void st1(void *p, long long i, float v) {
  reinterpret_cast<uint16_t *>(p)[i] = Elem<T>::from_float(v);
}
// Rounds through the 16-bit type, as a torch op on 16-bit tensors does.
template <typename T> __device__ __forceinline__ float r16(float v) {
  return Elem<T>::to_float(Elem<T>::from_float(v));
}

constexpr int kNormThreads = 256;

// One CTA per row.  h = x (+ residual, rounded to 16 bit); out = w * round16(h *
// rsqrt(mean(h^2) + eps)) with the statistics in FP32 (transformers LlamaRMSNorm).
template <typename T>
__global__ void __launch_bounds__(kNormThreads) rmsnorm_kernel(const void *x, const void *res, const void *w, void *out,
                                                               void *res_out, int cols, long long ld, float eps,
                                                               int pdl) {
  pdl_enter(pdl);
  const long long row = blockIdx.x;
  const void *xr = static_cast<const uint16_t *>(x) + row * ld;
  const void *rr = res ? static_cast<const uint16_t *>(res) + row * ld : nullptr;
  void *ro = res_out ? static_cast<void *>(static_cast<uint16_t *>(res_out) + row * ld) : nullptr;
  float ss = 0.f;
  for (int c = threadIdx.x; c < cols; c += kNormThreads) {
    float h = ld1<T>(xr, c);
    if (rr) h = r16<T>(h + ld1<T>(rr, c));
    if (ro) st1<T>(ro, c, h);
    ss = fmaf(h, h, ss);
  }
  __shared__ float red[kNormThreads / 32];
#pragma unroll
  for (int m = 16; m > 0; m >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, m);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int i = 0; i < kNormThreads / 32; ++i) tot += red[i];
  const float inv = rsqrtf(tot / (float)cols + eps);
  void *orow = static_cast<uint16_t *>(out) + row * (long long)cols;
  for (int c = threadIdx.x; c < cols; c += kNormThreads) {
    // Re-read h: from res_out when the add was fused (it may alias x or res).
    float h = ro ? ld1<T>(ro, c) : ld1<T>(xr, c);
    st1<T>(orow, c, ld1<T>(w, c) * r16<T>(h * inv));
  }
}

// Vectorized RMSNorm for rows whose buffers are 16-byte aligned and whose
// length is a multiple of 8: one CTA per row, each thread owning NV 16-byte
// vectors (8 elements each) of it.  Every thread issues all its loads (x,
// residual, weight) before using any, so a row costs one memory round trip
// instead of one per 256 elements; h stays in registers between the sum of
// squares and the output.  Same arithmetic as rmsnorm_kernel: h = x (+
// residual, rounded to 16 bit), statistics in FP32, out = w * round16(h * inv).
template <typename T, int NV>
__global__ void __launch_bounds__(kNormThreads) rmsnorm_vec_kernel(const void *x, const void *res, const void *w,
                                                                   void *out, void *res_out, int cols, long long ld,
                                                                   float eps, int pdl) {
  pdl_enter(pdl);
  const long long row = blockIdx.x;
  const int nvec = cols / 8;
  const uint4 *xr = reinterpret_cast<const uint4 *>(static_cast<const uint16_t *>(x) + row * ld);
  const uint4 *rr = res ? reinterpret_cast<const uint4 *>(static_cast<const uint16_t *>(res) + row * ld) : nullptr;
  const uint4 *wv = reinterpret_cast<const uint4 *>(w);
  uint4 hv[NV], wr[NV];
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const int v = threadIdx.x + j * kNormThreads;
    hv[j] = v < nvec ? xr[v] : make_uint4(0u, 0u, 0u, 0u);
    wr[j] = v < nvec ? wv[v] : make_uint4(0u, 0u, 0u, 0u);
  }
  if (rr) {
    uint4 rv[NV];
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      const int v = threadIdx.x + j * kNormThreads;
      rv[j] = v < nvec ? rr[v] : make_uint4(0u, 0u, 0u, 0u);
    }
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      uint32_t *h = reinterpret_cast<uint32_t *>(&hv[j]);
      const uint32_t *r = reinterpret_cast<const uint32_t *>(&rv[j]);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 a = Elem<T>::to_float2(h[e]), b = Elem<T>::to_float2(r[e]);
        h[e] = Elem<T>::pack2(a.x + b.x, a.y + b.y);  // rounded to 16 bit, as torch's add
      }
    }
    uint4 *ro = reinterpret_cast<uint4 *>(static_cast<uint16_t *>(res_out) + row * ld);
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      const int v = threadIdx.x + j * kNormThreads;
      if (v < nvec) ro[v] = hv[j];
    }
  }
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const uint32_t *h = reinterpret_cast<const uint32_t *>(&hv[j]);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 a = Elem<T>::to_float2(h[e]);
      ss = fmaf(a.x, a.x, ss);
      ss = fmaf(a.y, a.y, ss);
    }
  }
  __shared__ float red[kNormThreads / 32];
#pragma unroll
  for (int m = 16; m > 0; m >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, m);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int i = 0; i < kNormThreads / 32; ++i) tot += red[i];
  const float inv = rsqrtf(tot / (float)cols + eps);
  uint4 *orow = reinterpret_cast<uint4 *>(static_cast<uint16_t *>(out) + row * (long long)cols);
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const int v = threadIdx.x + j * kNormThreads;
    if (v >= nvec) continue;
    uint4 o;
    const uint32_t *h = reinterpret_cast<const uint32_t *>(&hv[j]);
    const uint32_t *wk = reinterpret_cast<const uint32_t *>(&wr[j]);
    uint32_t *ov = reinterpret_cast<uint32_t *>(&o);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 a = Elem<T>::to_float2(h[e]), ww = Elem<T>::to_float2(wk[e]);
      const float n0 = Elem<T>::to_float(Elem<T>::from_float(a.x * inv));
      const float n1 = Elem<T>::to_float(Elem<T>::from_float(a.y * inv));
      ov[e] = Elem<T>::pack2(ww.x * n0, ww.y * n1);
    }
    orow[v] = o;
  }
}

template <typename T>
cudaError_t launch_rmsnorm(cudaStream_t s, int rows, int cols, int pdl, const void *x, const void *res,
                           const void *w, void *out, void *res_out, long long ld, float eps) {
  const dim3 grid(rows), block(kNormThreads);
  const int nvec = cols / 8;
  const bool vec = cols % 8 == 0 && ld % 8 == 0 && nvec <= 8 * kNormThreads &&
                   ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(res) |
                     reinterpret_cast<uintptr_t>(w) | reinterpret_cast<uintptr_t>(out) |
                     reinterpret_cast<uintptr_t>(res_out)) & 15u) == 0;
  if (!vec) return launch_ex(rmsnorm_kernel<T>, grid, block, 0, s, 1, pdl, x, res, w, out, res_out, cols, ld, eps, pdl);
  if (nvec <= kNormThreads)
    return launch_ex(rmsnorm_vec_kernel<T, 1>, grid, block, 0, s, 1, pdl, x, res, w, out, res_out, cols, ld, eps, pdl);
  if (nvec <= 2 * kNormThreads)
    return launch_ex(rmsnorm_vec_kernel<T, 2>, grid, block, 0, s, 1, pdl, x, res, w, out, res_out, cols, ld, eps, pdl);
  if (nvec <= 4 * kNormThreads)
    return launch_ex(rmsnorm_vec_kernel<T, 4>, grid, block, 0, s, 1, pdl, x, res, w, out, res_out, cols, ld, eps, pdl);
  return launch_ex(rmsnorm_vec_kernel<T, 8>, grid, block, 0, s, 1, pdl, x, res, w, out, res_out, cols, ld, eps, pdl);
}

// One CTA per (sequence, head) of q, k and v, head_dim / 2 threads: for q and k,
// thread i rotates the pair (i, i + d/2) with cos/sin of position * inv_freq[i]
// rounded to 16 bit (transformers apply_rotary_pos_emb, default rotary
// embedding); v heads are copied, so all three outputs are contiguous.
template <typename T>
__global__ void rope_qk_kernel(const void *qkv, long long ld, const int32_t *pos, const float *inv_freq, void *q_out,
                               void *k_out, void *v_out, int q_heads, int kv_heads, int d, int pdl) {
  pdl_enter(pdl);
  const int heads = q_heads + 2 * kv_heads;
  const int b = blockIdx.x / heads;
  const int hh = blockIdx.x - b * heads;
  const int i = threadIdx.x;
  const int half = d / 2;
  if (i >= half) return;
  const long long src = (long long)b * ld + (long long)hh * d;
  const uint16_t *in = reinterpret_cast<const uint16_t *>(qkv);
  if (hh >= q_heads + kv_heads) {
    uint16_t *vo = reinterpret_cast<uint16_t *>(v_out) + ((long long)b * kv_heads + (hh - q_heads - kv_heads)) * d;
    vo[i] = in[src + i];
    vo[i + half] = in[src + i + half];
    return;
  }
  float o1, o2;
  rope_pair<T>(ld1<T>(qkv, src + i), ld1<T>(qkv, src + i + half), (float)pos[b] * inv_freq[i], o1, o2);
  void *dst;
  long long off;
  if (hh < q_heads) {
    dst = q_out;
    off = ((long long)b * q_heads + hh) * d;
  } else {
    dst = k_out;
    off = ((long long)b * kv_heads + (hh - q_heads)) * d;
  }
  st1<T>(dst, off + i, o1);
  st1<T>(dst, off + i + half, o2);
}

// out[r, c] = round16(silu(g)) * u with g = gu[r, c], u = gu[r, cols + c].
template <typename T>
__global__ void silu_mul_kernel(const void *gu, long long ld, void *out, int rows, int cols, int pdl) {
  pdl_enter(pdl);
  const long long n = (long long)rows * cols;
  for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < n; e += (long long)gridDim.x * blockDim.x) {
    const long long r = e / cols;
    const int c = (int)(e - r * cols);
    const float g = ld1<T>(gu, r * ld + c);
    const float u = ld1<T>(gu, r * ld + cols + c);
    const float sg = r16<T>(g / (1.0f + expf(-g)));
    st1<T>(out, e, sg * u);
  }
}

// RMSNorm whose input is the all-reduce of FP32 partials that every rank of a
// tensor-parallel group left in its own buffer (dak_linear_split_allreduce in
// publish-only mode).  Thread 0 waits, bounded, until every rank published the
// current call; then the row is read as sums over ranks with multimem.ld_reduce
// through the buffer's multicast address, 8 columns per thread, issued before
// any is used: as two 16-byte reads of 4 adjacent columns (VEC4, when the row
// and buffer are 16-byte aligned) or as 8 single-column reads.  Every column
// is summed over the ranks in FP32 by the switch either way.
// h = round16(round16(sum) + residual) is written back to the residual
// stream, and out = w * round16(h * rsqrt(mean(h^2) + eps)).
__device__ __forceinline__ float mm_ld_reduce_add(const float *p) {
  float v;
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.f32 %0, [%1];" : "=f"(v) : "l"(p));
  return v;
}
__device__ __forceinline__ float4 mm_ld_reduce_add_v4(const float *p) {
  float4 v;
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "l"(p));
  return v;
}
__device__ __forceinline__ uint32_t ld_acquire_sys_u32(const uint32_t *p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// One row is split over a cluster of kArCluster CTAs, so that every read of the
// row through the switch is in flight at once: each CTA handles cols /
// kArCluster columns with one batch of independent reads per thread, and the
// CTAs' sums of squares meet through distributed shared memory.
constexpr int kArCluster = 8;
constexpr int kArThreads = 128;
constexpr int kArPerThread = 8;  // columns per thread: cols <= kArCluster x 128 x 8 = 8192

__device__ __forceinline__ float ld_cluster_f32(uint32_t addr) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
  return v;
}

template <typename T, bool VEC4>
__global__ void __launch_bounds__(kArThreads) rmsnorm_ar_kernel(const float *mc, long long slot, long long ld,
                                                                const int *epoch, const uint32_t *flags, int world,
                                                                long long timeout_ns, int *status, void *res,
                                                                const void *w, void *out, int cols, float eps,
                                                                int pdl) {
  pdl_enter(pdl);  // the epoch below is advanced by the linear kernel before this one
  __shared__ int fail_s;
  __shared__ float red[kArThreads / 32];
  __shared__ float part;  // this CTA's sum of squares, read by the cluster
  const int k = (int)cluster_ctarank();
  const long long row = blockIdx.x / kArCluster;
  const int c_lo = (int)((long long)k * cols / kArCluster), c_hi = (int)((long long)(k + 1) * cols / kArCluster);
  const uint32_t e = (uint32_t)*reinterpret_cast<const volatile int *>(epoch);
  if (threadIdx.x == 0) {
    fail_s = 0;
    const unsigned long long t0 = globaltimer();
    for (int rk = 0; rk < world && !fail_s; ++rk)
      while ((int)(ld_acquire_sys_u32(flags + rk) - e) < 0) {
        if (globaltimer() - t0 > (unsigned long long)timeout_ns) {
          atomicCAS(status, 0, DAK_ERR_TIMEOUT);
          fail_s = 1;
          break;
        }
      }
  }
  __syncthreads();
  const bool ok = !fail_s;
  const float *src = mc + (long long)(e & 1u) * slot + row * ld;
  uint16_t *rrow = static_cast<uint16_t *>(res) + row * (long long)cols;
  // Column of this thread's u-th value: 4 adjacent columns per 16-byte read
  // (VEC4), else one column per read, threads adjacent.
  auto col_of = [&](int u) {
    return VEC4 ? c_lo + 4 * ((int)threadIdx.x + (u >> 2) * kArThreads) + (u & 3)
                : c_lo + (int)threadIdx.x + u * kArThreads;
  };
  float v[kArPerThread];
  if (VEC4) {
    // c_lo and c_hi are multiples of 4, so a group is wholly in or out.
#pragma unroll
    for (int g = 0; g < kArPerThread / 4; ++g) {
      const int c = col_of(4 * g);
      const float4 q = (ok && c < c_hi) ? mm_ld_reduce_add_v4(src + c) : make_float4(0.f, 0.f, 0.f, 0.f);
      v[4 * g] = q.x;
      v[4 * g + 1] = q.y;
      v[4 * g + 2] = q.z;
      v[4 * g + 3] = q.w;
    }
  } else {
#pragma unroll
    for (int u = 0; u < kArPerThread; ++u) {
      const int c = col_of(u);
      v[u] = (ok && c < c_hi) ? mm_ld_reduce_add(src + c) : 0.f;
    }
  }
  float ss = 0.f;
#pragma unroll
  for (int u = 0; u < kArPerThread; ++u) {
    const int c = col_of(u);
    if (ok && c < c_hi) {
      const float h = r16<T>(r16<T>(v[u]) + ld1<T>(rrow, c));
      v[u] = h;
      st1<T>(rrow, c, h);
      ss = fmaf(h, h, ss);
    }
  }
#pragma unroll
  for (int m = 16; m > 0; m >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, m);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
#pragma unroll
    for (int i = 0; i < kArThreads / 32; ++i) t += red[i];
    part = t;
  }
  // Every CTA's partial is written before any CTA reads them, and no CTA
  // leaves while a peer may still read its shared memory.
  cluster_sync_all();
  float tot = 0.f;
#pragma unroll
  for (int q = 0; q < kArCluster; ++q) tot += ld_cluster_f32(mapa_shared(smem_u32(&part), (uint32_t)q));
  cluster_sync_all();
  if (!ok) return;
  const float inv = rsqrtf(tot / (float)cols + eps);
  uint16_t *orow = static_cast<uint16_t *>(out) + row * (long long)cols;
#pragma unroll
  for (int u = 0; u < kArPerThread; ++u) {
    const int c = col_of(u);
    if (c < c_hi) st1<T>(orow, c, ld1<T>(w, c) * r16<T>(v[u] * inv));
  }
}

int check_dtype(int dtype) {
  if (dtype != DAK_DTYPE_F16 && dtype != DAK_DTYPE_BF16)
    return fail(DAK_ERR_UNSUPPORTED, "decode ops support float16 and bfloat16");
  return DAK_OK;
}

}  // namespace
}  // namespace dak

extern "C" int dak_rmsnorm(const void *x, const void *residual, const void *weight, void *out, void *residual_out,
                           int rows, int cols, int64_t ld, float eps, int dtype, void *stream) {
  using namespace dak;
  int st = check_dtype(dtype);
  if (st) return st;
  if (!x || !weight || !out || rows <= 0 || cols <= 0 || ld < cols)
    return fail(DAK_ERR_INVALID_ARG, "rmsnorm: x, weight, out and rows, cols > 0, ld >= cols are required");
  if ((residual == nullptr) != (residual_out == nullptr))
    return fail(DAK_ERR_INVALID_ARG, "rmsnorm: residual and residual_out come together");
  auto s = static_cast<cudaStream_t>(stream);
  const int pdl = decode_pdl_enabled() ? 1 : 0;
  const cudaError_t e =
      dtype == DAK_DTYPE_F16
          ? launch_rmsnorm<__half>(s, rows, cols, pdl, x, residual, weight, out, residual_out, (long long)ld, eps)
          : launch_rmsnorm<__nv_bfloat16>(s, rows, cols, pdl, x, residual, weight, out, residual_out, (long long)ld,
                                          eps);
  return cuda_status(e, "rmsnorm launch");
}

extern "C" int dak_rope_qk(const void *qkv, int64_t ld, const int32_t *positions, const float *inv_freq, void *q_out,
                           void *k_out, void *v_out, int batch, int q_heads, int kv_heads, int head_dim, int dtype,
                           void *stream) {
  using namespace dak;
  int st = check_dtype(dtype);
  if (st) return st;
  if (!qkv || !positions || !inv_freq || !q_out || !k_out || !v_out || batch <= 0 || q_heads <= 0 || kv_heads <= 0)
    return fail(DAK_ERR_INVALID_ARG, "rope_qk: all buffers and positive sizes are required");
  if (head_dim <= 0 || head_dim % 2 || head_dim > 1024)
    return fail(DAK_ERR_INVALID_ARG, "rope_qk: head_dim must be even and at most 1024");
  if (ld < (int64_t)(q_heads + 2 * kv_heads) * head_dim)
    return fail(DAK_ERR_INVALID_ARG, "rope_qk: qkv row stride below (q_heads + 2 kv_heads) x head_dim");
  auto s = static_cast<cudaStream_t>(stream);
  const int grid = batch * (q_heads + 2 * kv_heads);
  const int threads = ((head_dim / 2 + 31) / 32) * 32;
  const int pdl = decode_pdl_enabled() ? 1 : 0;
  const cudaError_t e =
      dtype == DAK_DTYPE_F16
          ? launch_ex(rope_qk_kernel<__half>, dim3(grid), dim3(threads), 0, s, 1, pdl, qkv, (long long)ld, positions,
                      inv_freq, q_out, k_out, v_out, q_heads, kv_heads, head_dim, pdl)
          : launch_ex(rope_qk_kernel<__nv_bfloat16>, dim3(grid), dim3(threads), 0, s, 1, pdl, qkv, (long long)ld,
                      positions, inv_freq, q_out, k_out, v_out, q_heads, kv_heads, head_dim, pdl);
  return cuda_status(e, "rope_qk launch");
}

extern "C" int dak_silu_mul(const void *gate_up, int64_t ld, void *out, int rows, int cols, int dtype, void *stream) {
  using namespace dak;
  int st = check_dtype(dtype);
  if (st) return st;
  if (!gate_up || !out || rows <= 0 || cols <= 0 || ld < 2 * (int64_t)cols)
    return fail(DAK_ERR_INVALID_ARG, "silu_mul: buffers, rows, cols > 0 and ld >= 2 cols are required");
  auto s = static_cast<cudaStream_t>(stream);
  const long long n = (long long)rows * cols;
  const int grid = (int)std::min<long long>((n + 255) / 256, 148 * 8);
  const int pdl = decode_pdl_enabled() ? 1 : 0;
  const cudaError_t e =
      dtype == DAK_DTYPE_F16
          ? launch_ex(silu_mul_kernel<__half>, dim3(grid), dim3(256), 0, s, 1, pdl, gate_up, (long long)ld, out, rows,
                      cols, pdl)
          : launch_ex(silu_mul_kernel<__nv_bfloat16>, dim3(grid), dim3(256), 0, s, 1, pdl, gate_up, (long long)ld,
                      out, rows, cols, pdl);
  return cuda_status(e, "silu_mul launch");
}

extern "C" int dak_rmsnorm_allreduce(const dak_allreduce_args *ar, void *residual, const void *weight, void *out,
                                     int rows, int cols, int64_t ld, float eps, int dtype, void *stream) {
  using namespace dak;
  int st = check_dtype(dtype);
  if (st) return st;
  if (!ar || !ar->mc_f32 || !ar->epoch || ar->world < 1 || ar->world > 8 || ar->rank < 0 || ar->rank >= ar->world ||
      !ar->flags[ar->rank])
    return fail(DAK_ERR_INVALID_ARG, "rmsnorm_allreduce: multicast all-reduce args with this rank's flags are required");
  if (!residual || !weight || !out || rows <= 0 || cols <= 0 || ld < cols || (long long)rows * ld > ar->slot_elems)
    return fail(DAK_ERR_INVALID_ARG, "rmsnorm_allreduce: residual, weight, out, rows, cols > 0 and rows x ld <= slot_elems");
  int *status = device_status_word();
  if (!status) return fail(DAK_ERR_CUDA, "no device status word");
  auto s = static_cast<cudaStream_t>(stream);
  const long long tns = ar->timeout_us * 1000;
  if (cols > kArCluster * kArThreads * kArPerThread)
    return fail(DAK_ERR_UNSUPPORTED, "rmsnorm_allreduce serves at most %d columns", kArCluster * kArThreads * kArPerThread);
  const int pdl = decode_pdl_enabled() ? 1 : 0;
  const dim3 grid((unsigned)rows * kArCluster), block(kArThreads);
  // 16-byte multicast reads need every row start, every CTA's first column
  // (cols / 8 apart) and both parity slots 16-byte aligned.
  const bool vec4 = cols % (4 * kArCluster) == 0 && ld % 4 == 0 && ar->slot_elems % 4 == 0 &&
                    (reinterpret_cast<uintptr_t>(ar->mc_f32) & 15u) == 0;
  auto launch = [&](auto kern) {
    return launch_ex(kern, grid, block, 0, s, kArCluster, pdl, (const float *)ar->mc_f32, (long long)ar->slot_elems,
                     (long long)ld, (const int *)ar->epoch, (const uint32_t *)ar->flags[ar->rank], ar->world, tns,
                     status, residual, weight, out, cols, eps, pdl);
  };
  cudaError_t e;
  if (dtype == DAK_DTYPE_F16)
    e = vec4 ? launch(rmsnorm_ar_kernel<__half, true>) : launch(rmsnorm_ar_kernel<__half, false>);
  else
    e = vec4 ? launch(rmsnorm_ar_kernel<__nv_bfloat16, true>) : launch(rmsnorm_ar_kernel<__nv_bfloat16, false>);
  if (e != cudaSuccess) return cuda_status(e, "rmsnorm_allreduce launch");
  return cuda_status(cudaGetLastError(), "rmsnorm_allreduce launch");
}
