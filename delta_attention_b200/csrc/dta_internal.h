// Host-side helpers shared by the C-ABI translation units (not exported).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

namespace dta {

// Record `e` as this thread's last CUDA error (dta_last_cuda_error), clear the
// runtime's pending error state, and return DTA_ERR_CUDA.
int fail_cuda(cudaError_t e);

// DTA_OK when the current device is sm_100 (its SM count in *sms), else
// DTA_ERR_UNSUPPORTED_DEVICE or DTA_ERR_CUDA.  Thread-safe; cached per device.
int check_device(int* sms);

// 4-D bf16 tensor map over (d, rows, heads, batch) with a 128-byte swizzle and
// a (64, box_rows, box_heads, 1) box; strides in elements.  DTA_OK or DTA_ERR_CUDA.
int encode_4d(CUtensorMap* map, const void* base, int d, long long rows, int heads, int batch, long long s_row,
              long long s_head, long long s_batch, int box_rows, int box_heads);

}  // namespace dta
