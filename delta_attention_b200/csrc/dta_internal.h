// Host-side helpers shared by the C-ABI translation units (not exported).
#pragma once

#include <cuda_runtime.h>

namespace dta {

// Record `e` as this thread's last CUDA error (dta_last_cuda_error), clear the
// runtime's pending error state, and return DTA_ERR_CUDA.
int fail_cuda(cudaError_t e);

// DTA_OK when the current device is sm_100 (its SM count in *sms), else
// DTA_ERR_UNSUPPORTED_DEVICE or DTA_ERR_CUDA.  Thread-safe; cached per device.
int check_device(int* sms);

}  // namespace dta
