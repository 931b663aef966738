// li4_internal.h -- host-side helpers shared by the C-ABI translation units.
#pragma once

#include <cuda_runtime.h>
#include <stdarg.h>
#include <stdint.h>

#include "../../include/llama_int4_b200.h"

namespace li4 {

// Record a formatted message for li4_last_error() and return `status`.
int set_error(int status, const char* fmt, ...);
// Clear the per-thread message (successful call).
void clear_error();
// Map a CUDA error to LI4_ERR_CUDA with context; LI4_OK if err == cudaSuccess.
int check_cuda(cudaError_t err, const char* what);
// SM count of the current device (cached per device ordinal).
int current_sm_count();
// Device error word of the communication kernels (li4_comm.cu); reset clears it.
int comm_device_errors(unsigned* flags, bool reset);
// Device error words of the decode program kernel (li4_program.cu); reset clears them.
int program_device_errors(unsigned* flags, bool reset);
// Device error word of the tensor-core GEMM (li4_gemm.cu); reset clears it.
int gemm_device_errors(unsigned* flags, bool reset);
// The GEMV device error words of the slab, register-rows, ring and program translation units.
int slab_device_errors(unsigned* flags, bool reset);
int rows_device_errors(unsigned* flags, bool reset);
int ring_device_errors(unsigned* flags, bool reset);
int program_gemv_device_errors(unsigned* flags, bool reset);
// Device error word of the argmax kernels (bit 6) and the poll limit of their key exchange.
int sample_device_errors(unsigned* flags, bool reset);
int sample_set_wait_limit(unsigned polls);
// Poll limit of the LI4_EPI_ALLREDUCE_RESIDUAL epilogue's waits (0 = default).
int gemv_set_ar_wait_limit(unsigned polls);
// Poll limit of the all-reduce flag waits (li4_comm.cu); 0 restores the default.
int comm_set_wait_limit(unsigned polls);
// Poll limit of the program's counter waits and an unmeetable-target offset (li4_program.cu).
int program_set_wait_limits(unsigned polls, unsigned extra);

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
inline bool is_pow2(int64_t v) { return v > 0 && (v & (v - 1)) == 0; }
inline int ilog2(int64_t v) { int r = 0; while ((int64_t(1) << r) < v) ++r; return r; }

}  // namespace li4
