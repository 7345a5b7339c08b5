// Host-side helpers shared by the C-ABI entry points (not part of the ABI).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace asb {

// Record a message for as_last_error() on this thread and return `code`.
int fail(int code, const char* fmt, ...);

// Check the launch of the kernel just issued; returns AS_OK or AS_ERR_CUDA.
int check_launch(const char* what);

// Device address of the current device's status word (set up once per device).
int* device_status_ptr();

// Size in bytes of one element of an AS_DTYPE_* type (0 for an unknown type).
int dtype_size(int dtype);

// cuTensorMapEncodeTiled resolved through the runtime's driver entry point
// (no link-time dependency on libcuda).  Returns AS_OK or an error code.
int encode_tensor_map(CUtensorMap* map, CUtensorMapDataType dtype, uint32_t rank,
                      void* base, const uint64_t* dims, const uint64_t* strides_bytes,
                      const uint32_t* box, CUtensorMapSwizzle swizzle);

// Number of SMs on the current device (cached per device).
int sm_count();

// Limit of every bounded mbarrier wait in the kernels launched from now on
// (as_set_wait_limit_ns; 2 s unless changed).
uint64_t wait_limit_ns();

// Test hook of as_debug_starve_next_launch: true (once) if the next launch of the
// attention kernel `kernel_bit` (AS_KERNEL_*) must issue no loads.
bool take_starve_flag(int kernel_bit);

}  // namespace asb
