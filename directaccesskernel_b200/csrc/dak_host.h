// dak_host.h - host-side declarations shared by the translation units of
// libdak_b200.so (not part of the public C ABI).
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include <algorithm>
#include <utility>

#include "dak_linear.cuh"

namespace dak {

// Records a failure for dak_last_error_message() and returns `code`.
int fail(int code, const char *fmt, ...);
// Maps a CUDA runtime error to DAK_ERR_CUDA with its text (or DAK_OK).
int cuda_status(cudaError_t e, const char *what);

// Identity of the CUDA context current on the calling thread (0 = none); unique
// for the life of the process.  Per-device state that holds device addresses
// or kernel attributes is set up again when it changes.
uint64_t current_context_id();
// Device address of the kernels' error word in the current context.
int *device_status_word();
// DAK_OK if `p` is memory of the current device or pinned host memory.
int check_gpu_accessible(const void *p, const char *what);

// Programmatic dependent launch of the decode-step kernels (RMSNorm, rotary,
// SiLU-gate, KV append, decode attention and its merge): on unless
// DAK_B200_NO_PDL=1.  Each of them is launched with programmatic stream
// serialization, waits for the previous kernel (griddepcontrol.wait) before it
// touches memory, and lets the next kernel be scheduled, so launches overlap
// the tail of the kernel before.
bool decode_pdl_enabled();

// cudaLaunchKernelEx with optional 1-D clusters (cluster > 1) and programmatic
// stream serialization (pdl).
template <typename... KArgs, typename... Args>
cudaError_t launch_ex(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream, int cluster,
                      bool pdl, Args &&...args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  int n = 0;
  if (cluster > 1) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = cluster;
    attr[n].val.clusterDim.y = 1;
    attr[n].val.clusterDim.z = 1;
    ++n;
  }
  if (pdl) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

// Shared-memory bytes and launch of the CUDA-core kernel for `ntok_tmpl`
// (1, 2, 4 or 8) tokens and dtype (DAK_DTYPE_F16 / _BF16).  With grid == 0
// nothing is launched and *max_clusters (if given) receives how many
// clusters of `cluster` CTAs can be resident at once.
size_t linear_core_smem_bytes(int ntok_tmpl, int red_slots);
int linear_core_stages(int ntok_tmpl, int red_slots);
cudaError_t launch_linear_core(const LinearParams &p, int ntok_tmpl, int dtype, int grid,
                               int cluster, size_t smem, cudaStream_t stream,
                               int *max_clusters = nullptr);

// Same for the tcgen05 kernel; `ntok_tmpl` is the UMMA N (multiple of 16).
size_t linear_mma_smem_bytes(int ntok_tmpl, int red_slots);
int linear_mma_stages(int ntok_tmpl, int ksplit);
cudaError_t launch_linear_mma(const LinearParams &p, int ntok_tmpl, int dtype, int grid,
                              int cluster, size_t smem, cudaStream_t stream,
                              int *max_clusters = nullptr);

// The wide tcgen05 kernel: 257..512 tokens per launch, each weight tile
// streamed once for both 256-token halves; no split-K, no clusters.  Its
// weight tile maps use boxes of 64 features x linear_wide_k_rows() K rows and
// its activation map boxes of 64 K x 256 tokens.  With `pair`, each CTA
// instead applies one 256-token row of the batch (grid row, p.tok_slices
// rows) to two 128-feature tiles at once.
size_t linear_wide_smem_bytes(bool pair);
int linear_wide_k_rows();
cudaError_t launch_linear_wide(const LinearParams &p, int dtype, int grid, size_t smem, cudaStream_t stream,
                               bool pair = false);
// Batches above 256 tokens of a layer with host-resident rows go to the wide
// kernel in chunks of up to 512 tokens.

// Sets, once per kernel and device, the kernel's dynamic shared-memory limit
// to the device's opt-in maximum and allows non-portable cluster sizes.  Every
// launch of the kernel, of any size, then fits the function's attributes, also
// when a captured graph node is launched again on its own.
cudaError_t prepare_kernel_attributes(const void *kern);

// Launch (or, with grid == 0, occupancy query) of a linear kernel: `grid`
// CTAs along x (times p.tok_slices rows of token slices along y), 1-D
// clusters along x, programmatic stream serialization when p.pdl is set.
template <typename Kern>
cudaError_t launch_linear_kernel(Kern kern, const LinearParams &p, int grid, int threads, int cluster,
                                 size_t smem, cudaStream_t stream, int *max_clusters) {
  cudaError_t e = prepare_kernel_attributes(reinterpret_cast<const void *>(kern));
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid > 0 ? grid : cluster, grid > 0 ? (unsigned)std::max(1, p.tok_slices) : 1u);
  cfg.blockDim = dim3(threads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = cluster;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = p.pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  if (grid <= 0) {
    int n = 0;
    e = cudaOccupancyMaxActiveClusters(&n, kern, &cfg);
    if (max_clusters) *max_clusters = n;
    return e;
  }
  return cudaLaunchKernelEx(&cfg, kern, p);
}

}  // namespace dak
