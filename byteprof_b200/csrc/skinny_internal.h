// Internal interface between the C-ABI entry point (skinny.cu) and the tensor-core kernels
// (skinny_tc.cu: bf16 weights; skinny_i8.cu: int8 weights).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace bp {

// Stream-K workspace layout, the same for every shape: kTcMaxTiles tile counters, then the partials. (A
// layout that depended on the tile count would let one shape's partials land on another shape's
// counters, which must stay zero between launches.)
constexpr int kTcMaxTiles = 8192;
constexpr size_t kTcCountersBytes = static_cast<size_t>(kTcMaxTiles) * 4;

// Bytes of zero-initialised workspace the tensor-core path needs for an N x K weight (0 if N or K is 0,
// or if the shape runs in cluster mode).
size_t skinny_tc_workspace_bytes(int N, int K, bool int8);

// Whether the tensor-core path takes this problem (16-byte aligned bases, ldx a multiple of 8,
// 1 <= M <= 16; K a multiple of 8 for bf16 weights, of 16 and at most 131072 for int8 weights).
bool skinny_tc_supported(const void* x, long long ldx, const void* w, int M, int N, int K, bool int8);

int launch_skinny_tc(const void* x, long long ldx, const void* w, const void* w_scale, void* y, long long ldy, int y_f32,
                     int M, int N, int K, bool int8, void* ws, size_t ws_bytes, cudaStream_t stream);

// int8 weights (skinny_i8.cu).
size_t skinny_i8_workspace_bytes(int N, int K);
bool skinny_i8_supported(const void* x, long long ldx, const void* w, int M, int N, int K);
int launch_skinny_i8(const void* x, long long ldx, const void* w, const void* w_scale, void* y, long long ldy, int y_f32,
                     int M, int N, int K, void* ws, size_t ws_bytes, cudaStream_t stream);

// Exact int8 weights on the CUDA cores for 1..4 activation rows (skinny_i8x.cu): bit-identical to the int8
// tensor-core kernel (the same fixed-point digits and exact integer sums), one launch, no workspace. Needs
// 16-byte aligned x and w, ldx a multiple of 8, K a multiple of 16 up to 131072, and at most
// kI8xMaxDigitBytes of digit planes per CTA.
constexpr size_t kI8xMaxDigitBytes = 64 * 1024;
bool skinny_i8x_supported(const void* x, long long ldx, const void* w, int M, int N, int K);
int launch_skinny_i8x(const void* x, long long ldx, const void* w, const void* w_scale, void* y, long long ldy, int y_f32,
                      int M, int N, int K, cudaStream_t stream);

// int4 group-128 weights on the tensor cores (skinny_i4tc.cu): workspace bytes for an N x K weight, whether
// the problem fits (16-byte aligned x, w, scale, zero; ldx a multiple of 8; N a multiple of 8; K a
// multiple of 128 up to 131072; 1 <= M <= 16), and the launch (prep kernel + main kernel).
size_t skinny_i4tc_workspace_bytes(int N, int K);
bool skinny_i4tc_supported(const void* x, long long ldx, const void* w, const void* scale, const void* zero, int M,
                           int N, int K);
int launch_skinny_i4tc(const void* x, long long ldx, const uint8_t* w, const void* scale, const void* zero, void* y,
                       long long ldy, int y_f32, int M, int N, int K, void* ws, size_t ws_bytes, cudaStream_t stream);

// Shared host helpers (skinny_tc.cu): a 2D tensor map with 128-byte swizzle, the SM count of the current
// device, and whether programmatic dependent launch is on (BP_DISABLE_PDL=1 turns it off).
int tc_encode_2d(CUtensorMap* map, CUtensorMapDataType dtype, const void* base, uint64_t inner, uint64_t outer,
                 uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer, CUtensorMapL2promotion promo);
// Any rank (1-5): dims and box innermost first, strides (bytes) of dims 1.. ; zero fill out of bounds.
int tc_encode(CUtensorMap* map, CUtensorMapDataType dtype, int rank, const void* base, const uint64_t* dims,
              const uint64_t* strides, const uint32_t* box, CUtensorMapSwizzle swizzle, CUtensorMapL2promotion promo);
int tc_sm_count();
bool tc_pdl_enabled();

// Reads and clears the device error words of all units (synchronising copies); each unit whose kernels
// can time out has its own word and reader.
unsigned int read_and_clear_device_errors();
unsigned int read_device_errors_tc();
unsigned int read_device_errors_i8();
unsigned int read_device_errors_i4tc();
unsigned int read_device_errors_glob();
unsigned int read_device_errors_loc();

}  // namespace bp
