// Host-side access to the driver's tensor-map encoder without linking the driver library.
//
// cuTensorMapEncodeTiled lives in libcuda, which only exists where an NVIDIA driver is
// installed.  Linking it would make the extension fail to load on machines without one
// (build hosts, CPU-only test runs).  The CUDA runtime hands out driver entry points at run
// time instead (cudaGetDriverEntryPoint); the pointer is looked up once per process.
#pragma once
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

namespace s0 {

inline PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return static_cast<PFN_cuTensorMapEncodeTiled_v12000>(nullptr);
    return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }();
  return fn;
}

}  // namespace s0
