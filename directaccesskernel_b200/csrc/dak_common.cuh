// dak_common.cuh - sm_100a building blocks shared by the DAK B200 kernels:
// mbarriers with bounded waits, TMA tile / bulk copies, cluster (DSMEM)
// addressing, L2 cache policies and the device-side error word.
//
// Every wait in these kernels is bounded: a wait that has not completed after
// kWaitTimeoutNs (measured on %globaltimer) records DAK_ERR_TIMEOUT in the
// status word, raises the CTA's abort flag and returns false.  Once the abort
// flag is up every later wait returns false at once, so the CTA runs through
// its remaining control flow (and its barriers) without waiting and exits.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/dak_b200.h"

namespace dak {

constexpr unsigned long long kWaitTimeoutNs = 4000000000ull;  // 4 s

// ------------------------------------------------------------- scalar types
template <typename T> struct Elem;
template <> struct Elem<__half> {
  static __device__ __forceinline__ float2 to_float2(uint32_t v) {
    __half2 h = *reinterpret_cast<__half2 *>(&v);
    return __half22float2(h);
  }
  static __device__ __forceinline__ float to_float(uint16_t v) {
    return __half2float(__ushort_as_half(v));
  }
  static __device__ __forceinline__ uint16_t from_float(float f) {
    return __half_as_ushort(__float2half_rn(f));
  }
  static __device__ __forceinline__ uint32_t pack2(float a, float b) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t *>(&h);
  }
  // lo += w.lo * x, hi += w.hi * x with 16-bit inputs and FP32 accumulation:
  // the mixed-precision FMA converts its 16-bit operands exactly and rounds
  // once, the same result as fmaf(float(w), float(x), acc).
  static __device__ __forceinline__ void fma_pair(float &lo, float &hi, uint32_t w2, uint16_t x) {
    asm("{\n\t.reg .b16 wl, wh;\n\tmov.b32 {wl, wh}, %2;\n\t"
        "fma.rn.f32.f16 %0, wl, %3, %0;\n\tfma.rn.f32.f16 %1, wh, %3, %1;\n\t}"
        : "+f"(lo), "+f"(hi) : "r"(w2), "h"(x));
  }
};
template <> struct Elem<__nv_bfloat16> {
  static __device__ __forceinline__ float2 to_float2(uint32_t v) {
    __nv_bfloat162 h = *reinterpret_cast<__nv_bfloat162 *>(&v);
    return __bfloat1622float2(h);
  }
  static __device__ __forceinline__ float to_float(uint16_t v) {
    return __bfloat162float(__ushort_as_bfloat16(v));
  }
  static __device__ __forceinline__ uint16_t from_float(float f) {
    return __bfloat16_as_ushort(__float2bfloat16_rn(f));
  }
  static __device__ __forceinline__ uint32_t pack2(float a, float b) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t *>(&h);
  }
  static __device__ __forceinline__ void fma_pair(float &lo, float &hi, uint32_t w2, uint16_t x) {
    asm("{\n\t.reg .b16 wl, wh;\n\tmov.b32 {wl, wh}, %2;\n\t"
        "fma.rn.f32.bf16 %0, wl, %3, %0;\n\tfma.rn.f32.bf16 %1, wh, %3, %1;\n\t}"
        : "+f"(lo), "+f"(hi) : "r"(w2), "h"(x));
  }
};

// Rotary embedding of the pair (x1, x2) = (x[i], x[i + d/2]) by the angle
// position * inv_freq[i], with cos, sin, every product and every sum rounded to
// the 16-bit type, as transformers' apply_rotary_pos_emb computes it on 16-bit
// tensors: o1 = x1 c + (-x2) s, o2 = x2 c + x1 s.
template <typename T>
__device__ __forceinline__ void rope_pair(float x1, float x2, float angle, float &o1, float &o2) {
  auto r16 = [](float v) { return Elem<T>::to_float(Elem<T>::from_float(v)); };
  const float c = r16(cosf(angle)), s = r16(sinf(angle));
  o1 = r16(r16(x1 * c) + r16(-x2 * s));
  o2 = r16(r16(x2 * c) + r16(x1 * s));
}

// ---------------------------------------------------------------- addresses
__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ unsigned long long globaltimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// Address of the same shared-memory variable in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}

__device__ __forceinline__ void cluster_arrive() {
  asm volatile("barrier.cluster.arrive.release;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() {
  asm volatile("barrier.cluster.wait.acquire;" ::: "memory");
}
__device__ __forceinline__ void cluster_sync_all() {
  cluster_arrive();
  cluster_wait();
}
// Arrival without release semantics: the thread's earlier writes are not made
// visible to the cluster first, so it does not wait for outstanding global
// stores (which the end of the kernel orders anyway).
__device__ __forceinline__ void cluster_arrive_relaxed() {
  asm volatile("barrier.cluster.arrive.relaxed;" ::: "memory");
}
// Last barrier of a cluster before its CTAs exit: no CTA leaves while a peer
// may still write to its shared memory.  Threads whose last act was a write to
// a peer's shared memory (`remote`) arrive with release semantics, so that
// write lands before the peer can leave; the others arrive relaxed.
__device__ __forceinline__ void cluster_exit_sync(bool remote) {
  if (remote)
    cluster_arrive();
  else
    cluster_arrive_relaxed();
  cluster_wait();
}

// Named barrier over `count` threads (warp multiples), id 1..15.
__device__ __forceinline__ void named_sync(int id, int count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// ----------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}
// Arrive on an mbarrier of another CTA of the cluster (address from mapa),
// releasing this thread's prior writes at cluster scope.
__device__ __forceinline__ void mbar_arrive_remote(uint32_t remote_bar) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(remote_bar)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ bool mbar_try_wait_cluster(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Per-CTA abort state shared by the bounded waits.
struct WaitCtx {
  volatile int *abort;  // shared-memory flag of this CTA
  int *status;          // device status word (global)
};

__device__ __forceinline__ void record_error(const WaitCtx &w, int code) {
  *w.abort = 1;
  atomicCAS(w.status, 0, code);
}

template <bool kClusterScope>
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, const WaitCtx &w,
                                          unsigned long long timeout_ns = kWaitTimeoutNs) {
  auto probe = [&]() {
    return kClusterScope ? mbar_try_wait_cluster(bar, parity) : mbar_try_wait(bar, parity);
  };
  if (*w.abort) return false;
  if (probe()) return true;
  const unsigned long long t0 = globaltimer();
  uint32_t n = 0;
  while (true) {
    if (probe()) return true;
    if ((++n & 15u) == 0) {
      if (*w.abort) return false;
      if (globaltimer() - t0 > timeout_ns) {
        record_error(w, DAK_ERR_TIMEOUT);
        return false;
      }
    }
  }
}

// ------------------------------------------------------------ L2 policies
__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t l2_policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// --------------------------------------------------------------------- TMA
// 2-D tiled tensor load into this CTA's shared memory, completing on `bar`.
// No multicast form is used anywhere in this code base.
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap *map, int c0, int c1,
                                            uint32_t bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      ".L2::cache_hint [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(bar), "l"(policy)
      : "memory");
}

// 1-D bulk copy global -> shared (16-byte aligned addresses, size % 16 == 0).
__device__ __forceinline__ void bulk_load(uint32_t dst, const void *src, uint32_t bytes,
                                          uint32_t bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1], %2, [%3], %4;" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(bar), "l"(policy)
      : "memory");
}

__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap *map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// --------------------------------------------------- distributed shared mem
__device__ __forceinline__ void st_cluster_v4(uint32_t addr, float a, float b, float c, float d) {
  asm volatile("st.shared::cluster.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "f"(a), "f"(b),
               "f"(c), "f"(d)
               : "memory");
}

// ------------------------------------------- programmatic dependent launch
// Wait until the grids this launch depends on have completed and their
// memory is visible (no-op when the launch has no programmatic dependency).
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
// Let the next kernel of the stream be scheduled once every CTA of this grid
// has executed this (or exited).
__device__ __forceinline__ void griddep_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Entry of a decode-step kernel (norms, rotary, SiLU-gate, KV append,
// attention, merge): when launched with programmatic stream serialization
// (`pdl` set), every thread waits for the previous kernel of the stream before
// touching memory, and the next kernel may then be scheduled.
__device__ __forceinline__ void pdl_enter(int pdl) {
  if (pdl) {
    griddep_wait();
    griddep_launch_dependents();
  }
}

__device__ __forceinline__ int lane_id() { return threadIdx.x & 31; }
__device__ __forceinline__ int warp_id() { return threadIdx.x >> 5; }

}  // namespace dak
