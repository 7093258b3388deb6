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

// SM count of the current device (cached per device).  Also rejects devices
// that are not compute capability 10.0.
int device_sm_count(int* sms);

}  // namespace nvfp4
