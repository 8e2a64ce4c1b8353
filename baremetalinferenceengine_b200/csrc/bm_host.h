// Host-side helpers shared by the C ABI entry points: error reporting into a
// thread-local message, launch checks and per-device launch sizing.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "bm_layer_ops.h"

namespace bm {

// Records a message for bm_last_error_message() and returns `status`.
int fail(int status, const char* fmt, ...) __attribute__((format(printf, 2, 3)));

// Clears the thread's last error message.
void clear_error();

// Returns BM_OK, or BM_ERR_CUDA with the launch error of `what` recorded.
int check_launch(const char* what);

// Streaming multiprocessors of the current device (cached per device).
int sm_count();

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

inline int dtype_size(bm_dtype_t dt) { return dt == BM_F32 ? 4 : 2; }

inline bool valid_dtype(int dt) { return dt == BM_F32 || dt == BM_BF16; }

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

}  // namespace bm
