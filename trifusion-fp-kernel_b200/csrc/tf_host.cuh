// Host-side helpers shared by the C-ABI translation units (defined in tf_api.cu).
#pragma once

#include <cuda_runtime.h>

namespace tf {

// Last CUDA error text recorded by this thread.
extern thread_local char g_last_error[256];
// TF_OK when the current device is an sm_100 GPU (cached per device).
int check_device();
// TF_OK, or TF_ERR_LAUNCH with the error text recorded (cudaGetLastError).
int launch_status();
// Number of SMs of the current device (cached per device).
int sm_count();

}  // namespace tf
