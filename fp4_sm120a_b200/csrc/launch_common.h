// Host-side helpers shared by the launchers: status mapping, cached device
// properties.
#pragma once

#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

#include "nvfp4_b200.h"

namespace nvfp4 {

// Records the CUDA error for nvfp4_last_cuda_error() and maps it to a status.
int cuda_status(cudaError_t e);

// Global amax of `nbytes` (a multiple of 16) of bf16 at x (16-byte aligned)
// plus `ntail` (< 8) trailing values at tail, folded into *out_bits (fp32 bits,
// which the caller has zeroed) by the bulk-copy amax kernel.
int amax_bulk_launch(const void* x, size_t nbytes, const uint16_t* tail, int ntail,
                     uint32_t* out_bits, cudaStream_t stream);

// SM count of the current device (cached per device).  Also rejects devices
// that are not compute capability 10.0.
int device_sm_count(int* sms);

}  // namespace nvfp4
