// Host side of the TMA tensor maps: cuTensorMapEncodeTiled, resolved once per
// process through the runtime's driver entry point query.
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <mutex>

#include "common.cuh"

namespace lnet {

inline int tensor_map_encoder(PFN_cuTensorMapEncodeTiled_v12000 *out) {
  static PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void *fn = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  });
  if (!encode) return fail(LNET_ERR_CUDA, "cuTensorMapEncodeTiled is not available");
  *out = encode;
  return LNET_OK;
}

}  // namespace lnet
