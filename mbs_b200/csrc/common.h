// Host-side helpers shared by the kernels of libmbs_gemm_kernel.so: status
// reporting, device queries and TMA tensor-map encoding.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

#include "../../include/mbs_gemm_a4w4.h"

namespace mbs {

// Records a detail message for mbs_last_error_message() and returns `status`.
int fail(int status, const char* fmt, ...);
// Clears the last message (called at the start of every entry point).
void clear_error();

// Maps a CUDA error to MBS_ERR_CUDA with its name in the message.
int cuda_fail(cudaError_t e, const char* what);

struct DeviceInfo
{
    int device;
    int num_sms;
    int cc_major, cc_minor;
    size_t max_smem_optin;
};

// Current device, checked to be sm_100 (B200 family).  Returns MBS_OK or an error.
int current_device(DeviceInfo* info);

// Device-global sticky error word (MBS_ERR_DEVICE_TIMEOUT when a wait ran out).
unsigned* device_error_word(int device);

// Count of device errors cleared through mbs_device_error(..., reset=1).  A
// launch that stopped on a device error may leave stream-K flags set, so
// library-owned workspaces clear their flags when this has moved on.
unsigned long long device_error_epoch();

// cuTensorMapEncodeTiled through the runtime's driver entry point (no -lcuda).
int encode_tmap(CUtensorMap* map, CUtensorMapDataType dtype, int rank, void* base,
                const uint64_t* dims, const uint64_t* strides_bytes /* rank-1 entries */,
                const uint32_t* box, CUtensorMapSwizzle swizzle);

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

inline int round_up(int x, int m) { return (x + m - 1) / m * m; }

inline int scale_n_pad(int K) { return round_up((K + 31) / 32, 8); }

}  // namespace mbs
