// Host-side helpers shared by the C-ABI entry points: tensor-map encoding
// through the driver entry point (no -lcuda link), argument checks and the
// once-per-device shared-memory attribute setup.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>
#include <stdint.h>
#include <stdlib.h>

#include <mutex>
#include <set>
#include <utility>

#include "../../include/sa3b200.h"

namespace sa3 {

inline PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// 2-D tiled tensor map over a row-major [rows, cols] view with the 128-byte
// swizzle. box_cols * elem_bytes must be <= 128. Out-of-range elements of a
// box read as zero.
inline int make_tmap_2d(CUtensorMap* m, const void* base, CUtensorMapDataType dt, int elem_bytes, uint64_t cols,
                        uint64_t rows, uint64_t row_stride_elems, uint32_t box_cols, uint32_t box_rows,
                        CUtensorMapSwizzle swz = CU_TENSOR_MAP_SWIZZLE_128B) {
  auto fn = encode_fn();
  if (!fn) return SA3_ERR_LAUNCH;
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0) return SA3_ERR_ALIGN;
  if ((row_stride_elems * elem_bytes) % 16 != 0) return SA3_ERR_ALIGN;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {row_stride_elems * (uint64_t)elem_bytes};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(m, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? SA3_OK : SA3_ERR_LAUNCH;
}

inline int launch_status() {
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? SA3_OK : SA3_ERR_LAUNCH;
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

// Programmatic dependent launch for the hot kernels (every one of them calls grid_dep_wait()
// before touching global memory). SA3_PDL=0 in the environment turns it off.
inline bool pdl_enabled() {
  static const bool on = [] {
    const char* e = getenv("SA3_PDL");
    return !(e && e[0] == '0');
  }();
  return on;
}

// In-place fp32 residual GEMM epilogues add their result into C with TMA reduce-add (L2 does the
// read-modify-write) instead of loading the residual through the SM. SA3_RESIDUAL_REDUCE=0 selects
// the load / combine / store path.
inline bool sa3_residual_reduce_enabled() {
  static const bool on = [] {
    const char* e = getenv("SA3_RESIDUAL_REDUCE");
    return !(e && e[0] == '0');
  }();
  return on;
}

// cudaLaunchKernelEx with programmatic stream serialisation and, for cluster > 1, a 1-D cluster.
template <typename... KArgs, typename... Args>
inline int launch_ex(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, int cluster,
                     Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  int n = 0;
  if (pdl_enabled()) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  if (cluster > 1) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = cluster;
    attr[n].val.clusterDim.y = 1;
    attr[n].val.clusterDim.z = 1;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...) == cudaSuccess ? SA3_OK : SA3_ERR_LAUNCH;
}

// Raise the dynamic shared-memory limit of `func` once per device, so later
// calls (including those made during CUDA-graph stream capture) only launch.
template <typename F>
inline int ensure_smem(F func, int bytes) {
  static std::mutex mu;
  static std::set<std::pair<const void*, int>> done;  // (kernel, device) pairs already configured
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return SA3_ERR_LAUNCH;
  const auto key = std::make_pair(reinterpret_cast<const void*>(func), dev);
  std::lock_guard<std::mutex> g(mu);
  if (done.count(key)) return SA3_OK;
  if (cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) != cudaSuccess)
    return SA3_ERR_LAUNCH;
  done.insert(key);
  return SA3_OK;
}

}  // namespace sa3
