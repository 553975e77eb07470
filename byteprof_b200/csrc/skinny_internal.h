// Internal interface between the C-ABI entry point (skinny.cu) and the tensor-core kernel (skinny_tc.cu).
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>

namespace bp {

// Bytes of zero-initialised workspace the tensor-core path needs for an N x K weight (0 if N or K is 0,
// or if the shape runs in cluster mode).
size_t skinny_tc_workspace_bytes(int N, int K, bool int8);

// Whether the tensor-core path takes this problem (16-byte aligned bases, ldx a multiple of 8,
// 1 <= M <= 16, K a multiple of 8 for bf16 and of 128 for int8 weights).
bool skinny_tc_supported(const void* x, long long ldx, const void* w, int M, int N, int K, bool int8);

int launch_skinny_tc(const void* x, long long ldx, const void* w, const void* w_scale, void* y, long long ldy, int y_f32,
                     int M, int N, int K, bool int8, void* ws, size_t ws_bytes, cudaStream_t stream);

// Reads and clears the device error word (synchronising copy).
unsigned int read_and_clear_device_errors();

}  // namespace bp
