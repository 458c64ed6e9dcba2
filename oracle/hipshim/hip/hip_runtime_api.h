// CPU SIMT shim (test infrastructure): the HIP runtime types the reference's
// routed ABI header names.  See hip_runtime.h.
#pragma once
#include <stddef.h>
typedef int hipError_t;
enum { hipSuccess = 0, hipErrorInvalidValue = 1 };
typedef void* hipStream_t;
