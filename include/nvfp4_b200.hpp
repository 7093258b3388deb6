// nvfp4_b200.hpp -- C++ host mirror of the reference's launcher templates on
// top of the C ABI (include/nvfp4_b200.h).
//
//   nvfp4_b200::rht_gemm_ntt_w_sfc<TA, TB, TC, TSFC, SR, FM>(m, n, A, B, C, SFC,
//       global_amax, rng_state, sm_count, stream, k_tile_size = 2048)
//     replaces rht_gemm/te_ref/hadamard_transform_cast_fusion_core.inc:513-644
//   nvfp4_b200::rht_gemm_ttt_wrapper<...>(..., k_tile_size = 1024)
//     replaces core.inc:648-678
//
// Same names, template flags, positional arguments and defaults.  Element
// types are only checked for size (bf16 = 2 bytes; FP4 and E4M3 buffers are
// byte buffers), so cutlass/cute or CUDA types can be passed unchanged.
// Like the reference's NVTE_CHECK (te_ref/stubs/common/common.h:17-33), a
// failed check prints the reason and aborts; use the C ABI directly to get a
// status code instead.
#pragma once

#include <cstdio>
#include <cstdlib>
#include <cuda_runtime.h>

#include "nvfp4_b200.h"

namespace nvfp4_b200 {

inline void check_status(int status, const char* what) {
  if (status != NVFP4_OK) {
    std::fprintf(stderr, "%s failed: %s\n", what, nvfp4_status_string(status));
    std::abort();
  }
}

template <typename TA, typename TB, typename TC, typename TSFC, bool kEnableStochasticRounding = false,
          bool kUseFastMath = false>
void rht_gemm_ntt_w_sfc(int m, int n, TA const* A, TB const* B, TC* C, TSFC* SFC,
                        float const* global_amax, const size_t* rng_state, uint32_t sm_count,
                        cudaStream_t stream, int k_tile_size = 2048) {
  static_assert(sizeof(TA) == 2 && sizeof(TB) == 2, "A and B are bf16");
  check_status(nvfp4_rht_gemm_ntt_w_sfc(m, n, A, B, C, SFC, global_amax, rng_state, sm_count,
                                        reinterpret_cast<nvfp4_stream_t>(stream), k_tile_size,
                                        kEnableStochasticRounding, kUseFastMath),
               "rht_gemm_ntt_w_sfc");
}

template <typename TA, typename TB, typename TC, typename TSFC, bool kEnableStochasticRounding = false,
          bool kUseFastMath = false>
void rht_gemm_ttt_wrapper(int m, int n, TA const* A, TB const* B, TC* C, TSFC* SFC,
                          float const* global_amax, const size_t* rng_state, uint32_t sm_count,
                          cudaStream_t stream, int k_tile_size = 1024) {
  rht_gemm_ntt_w_sfc<TA, TB, TC, TSFC, kEnableStochasticRounding, kUseFastMath>(
      n, m, A, B, C, SFC, global_amax, rng_state, sm_count, stream, k_tile_size);
}

}  // namespace nvfp4_b200
