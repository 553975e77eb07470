// Skinny weight-only linear y[M, N] = x[M, K] . W[N, K]^T for M = 1..16 rows per launch, bf16 or int8
// weights (per-output-channel bf16 scale), fp32 accumulation, bf16 or fp32 output.
//
// Reference: byteprof/optim/skinny.py:35-166 (_skinny_kernel MODE 0/1, _split_reduce, _launch,
// skinny_mm) and byteprof/quant/triton_int8.py:15-47 (_gemv_int8, gemv_int8).
//
// B200 design (CUDA-core streaming path):
//  * Each warp owns R output rows and one K range. Lanes read 16 contiguous bytes of every row per
//    step (512 contiguous bytes per row per warp step), through a U-deep register pipeline of
//    `ld.global.nc.L1::no_allocate` loads carrying an L2 evict-first policy, so (U-1)*R 16-byte
//    loads per lane are in flight while the previous step is multiplied.
//  * int8 weights are widened to exact fp32 in registers (byte permute into the mantissa of 2^23,
//    one subtract); the per-row scale is applied once to the final sum.
//  * The M activation rows are read through L1 (every warp of a CTA re-reads the same slice).
//  * Split-K: the K ranges of one row tile form a thread-block cluster of S <= 8 CTAs. Partial sums
//    meet in shared memory and are added through distributed shared memory in split order
//    0..S-1, so the result is deterministic and no global workspace or second launch is needed
//    (the reference writes fp32 partials to a workspace and reduces them in a second kernel,
//    skinny.py:79-90, 125-129).
#include <cooperative_groups.h>

#include "bp_common.cuh"
#include "skinny_internal.h"

namespace cg = cooperative_groups;

namespace bp {
namespace {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;

struct SkinnyArgs {
  const void* x;  // bf16 or fp32 (the kernel's XT)
  long long ldx;
  const void* w;
  const __nv_bfloat16* scale;  // int8 only: [N]
  void* y;
  long long ldy;
  int y_f32;
  int N, K;
  int k_chunk;  // K elements per split (a multiple of the warp step, except for the last split)
};

template <typename WT>
struct WTraits;
template <>
struct WTraits<__nv_bfloat16> {
  static constexpr int EPL = 8;  // elements per 16-byte load
};
template <>
struct WTraits<int8_t> {
  static constexpr int EPL = 16;
};

// 16 bytes of weights -> EPL exact fp32 values.
__device__ __forceinline__ void unpack_w(const uint4& v, float (&f)[8]) {
  f[0] = bf16lo(v.x); f[1] = bf16hi(v.x);
  f[2] = bf16lo(v.y); f[3] = bf16hi(v.y);
  f[4] = bf16lo(v.z); f[5] = bf16hi(v.z);
  f[6] = bf16lo(v.w); f[7] = bf16hi(v.w);
}

// Signed byte q -> fp32 q: flip the sign bit (u = q + 128), place u in the low mantissa byte of
// 2^23 (exact: 2^23 + u), subtract 2^23 + 128.
__device__ __forceinline__ void unpack_w(const uint4& v, float (&f)[16]) {
  const uint32_t words[4] = {v.x ^ 0x80808080u, v.y ^ 0x80808080u, v.z ^ 0x80808080u, v.w ^ 0x80808080u};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
#pragma unroll
    for (int b = 0; b < 4; ++b)
      f[4 * j + b] = __uint_as_float(__byte_perm(words[j], 0x4B000000u, 0x7540u | b)) - 8388736.0f;
  }
}

template <int EPL>
__device__ __forceinline__ void load_x(const float* p, float (&f)[EPL]) {
#pragma unroll
  for (int h = 0; h < EPL / 4; ++h) {
    const float4 v = __ldg(reinterpret_cast<const float4*>(p) + h);
    f[4 * h + 0] = v.x; f[4 * h + 1] = v.y; f[4 * h + 2] = v.z; f[4 * h + 3] = v.w;
  }
}

template <int EPL>
__device__ __forceinline__ void load_x(const __nv_bfloat16* p, float (&f)[EPL]) {
#pragma unroll
  for (int h = 0; h < EPL / 8; ++h) {
    const uint4 v = ldg16(p + 8 * h);
    f[8 * h + 0] = bf16lo(v.x); f[8 * h + 1] = bf16hi(v.x);
    f[8 * h + 2] = bf16lo(v.y); f[8 * h + 3] = bf16hi(v.y);
    f[8 * h + 4] = bf16lo(v.z); f[8 * h + 5] = bf16hi(v.z);
    f[8 * h + 6] = bf16lo(v.w); f[8 * h + 7] = bf16hi(v.w);
  }
}

__device__ __forceinline__ float load_w1(const __nv_bfloat16* p) { return __bfloat162float(*p); }
__device__ __forceinline__ float load_w1(const float* p) { return *p; }
__device__ __forceinline__ float load_w1(const int8_t* p) { return static_cast<float>(*p); }

template <typename WT>
__device__ __forceinline__ float row_scale(const SkinnyArgs& a, int row) {
  if constexpr (sizeof(WT) == 1) return __bfloat162float(a.scale[row]);
  return 1.0f;
}

__device__ __forceinline__ void store_y(const SkinnyArgs& a, int m, int row, float v) {
  if (a.y_f32)
    static_cast<float*>(a.y)[m * a.ldy + row] = v;
  else
    static_cast<__nv_bfloat16*>(a.y)[m * a.ldy + row] = __float2bfloat16_rn(v);
}

template <typename WT, int M, int R, int U, bool VEC, typename XT>
__global__ void __launch_bounds__(kThreads) skinny_fma_kernel(const SkinnyArgs a) {
  constexpr int EPL = WTraits<WT>::EPL;
  constexpr int KW = VEC ? 32 * EPL : 32;  // K elements covered by one warp step
  __shared__ float part[kWarps * R * M];    // split-K partial sums of this CTA

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row0 = (blockIdx.x * kWarps + warp) * R;
  const int kb = blockIdx.y * a.k_chunk;
  const int ke = min(a.K, kb + a.k_chunk);
  const WT* __restrict__ w = static_cast<const WT*>(a.w);
  const XT* __restrict__ x = static_cast<const XT*>(a.x);

  pdl_launch_dependents();

  float acc[R][M];
#pragma unroll
  for (int r = 0; r < R; ++r)
#pragma unroll
    for (int m = 0; m < M; ++m) acc[r][m] = 0.0f;

  bool rv[R];
  const WT* wr[R];
#pragma unroll
  for (int r = 0; r < R; ++r) {
    rv[r] = row0 + r < a.N;
    wr[r] = w + static_cast<long long>(rv[r] ? row0 + r : 0) * a.K;
  }

  if constexpr (VEC) {
    const uint64_t pol = l2_evict_first_policy();
    uint4 buf[U][R];
    const int k0 = kb + lane * EPL;
#pragma unroll
    for (int u = 0; u < U - 1; ++u) {
      const int k = k0 + u * KW;
#pragma unroll
      for (int r = 0; r < R; ++r) buf[u][r] = (rv[r] && k < ke) ? ldg_stream16(wr[r] + k, pol) : make_uint4(0, 0, 0, 0);
    }
    pdl_wait_prior_grids();  // the weights above are constants; x may come from the kernel before
    for (int kk = k0; kk < ke; kk += U * KW) {
#pragma unroll
      for (int u = 0; u < U; ++u) {
        {  // refill the slot consumed one step ago with the step U-1 ahead
          const int kn = kk + (u + U - 1) * KW;
#pragma unroll
          for (int r = 0; r < R; ++r)
            buf[(u + U - 1) % U][r] = (rv[r] && kn < ke) ? ldg_stream16(wr[r] + kn, pol) : make_uint4(0, 0, 0, 0);
        }
        const int k = kk + u * KW;
        if (k < ke) {
          float xf[M][EPL];
#pragma unroll
          for (int m = 0; m < M; ++m) load_x<EPL>(x + m * a.ldx + k, xf[m]);
#pragma unroll
          for (int r = 0; r < R; ++r) {
            float wf[EPL];
            unpack_w(buf[u][r], wf);
#pragma unroll
            for (int m = 0; m < M; ++m)
#pragma unroll
              for (int e = 0; e < EPL; ++e) acc[r][m] = fmaf(wf[e], xf[m][e], acc[r][m]);
          }
        }
      }
    }
  } else {
    // Element-wise path for rows that are not 16-byte aligned (odd K): correctness, not speed.
    pdl_wait_prior_grids();
    for (int k = kb + lane; k < ke; k += 32) {
      float xf[M];
#pragma unroll
      for (int m = 0; m < M; ++m) xf[m] = load_w1(x + m * a.ldx + k);
#pragma unroll
      for (int r = 0; r < R; ++r) {
        const float wv = rv[r] ? load_w1(wr[r] + k) : 0.0f;
#pragma unroll
        for (int m = 0; m < M; ++m) acc[r][m] = fmaf(wv, xf[m], acc[r][m]);
      }
    }
  }

  // Sum each accumulator over the 32 lanes (butterfly: every lane ends with every sum).
#pragma unroll
  for (int r = 0; r < R; ++r)
#pragma unroll
    for (int m = 0; m < M; ++m) {
      float v = acc[r][m];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
      acc[r][m] = v;
    }

  if (gridDim.y == 1) {
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
      for (int m = 0; m < M; ++m)
        if (((r * M + m) & 31) == lane && rv[r]) store_y(a, m, row0 + r, acc[r][m] * row_scale<WT>(a, row0 + r));
    return;
  }

  // Split-K: the CTAs of one row tile form a cluster along y; rank s holds the partial of split s.
  if (lane == 0) {
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
      for (int m = 0; m < M; ++m) part[(warp * R + r) * M + m] = acc[r][m];
  }
  cg::cluster_group cluster = cg::this_cluster();
  cluster.sync();
  const int S = gridDim.y;
  const int rank = static_cast<int>(cluster.block_rank());
  const int tile_row0 = blockIdx.x * kWarps * R;
  for (int e = rank + S * threadIdx.x; e < kWarps * R * M; e += S * kThreads) {
    const int rr = e / M, m = e - rr * M;
    const int row = tile_row0 + rr;
    if (row >= a.N) continue;
    float s = 0.0f;
    for (int q = 0; q < S; ++q) s += cluster.map_shared_rank(part, q)[e];
    store_y(a, m, row, s * row_scale<WT>(a, row));
  }
  cluster.sync();  // keep this CTA's partials alive until every peer has read them
}

// ---- host side ---------------------------------------------------------------------------------

int g_sm_count[64] = {0};

int sm_count() {
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return 148;
  if (g_sm_count[dev] == 0) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    g_sm_count[dev] = n > 0 ? n : 148;
  }
  return g_sm_count[dev];
}

template <typename WT, int M>
struct Tile;  // rows per warp R and pipeline depth U per weight type and row count
template <int M>
struct Tile<__nv_bfloat16, M> {
  static constexpr int R = M <= 4 ? 4 : (M <= 8 ? 2 : 1);
  static constexpr int U = M <= 8 ? 3 : 4;
};
template <int M>
struct Tile<int8_t, M> {
  static constexpr int R = M <= 2 ? 4 : (M <= 8 ? 2 : 1);
  static constexpr int U = M <= 4 ? 3 : 2;
};

template <typename WT, int M, typename XT>
int launch_rows(SkinnyArgs a, bool vec, cudaStream_t st) {
  constexpr int R = Tile<WT, M>::R;
  constexpr int U = Tile<WT, M>::U;
  constexpr int EPL = WTraits<WT>::EPL;
  const int kw = vec ? 32 * EPL : 32;
  const int row_tiles = (a.N + kWarps * R - 1) / (kWarps * R);
  const int ksteps = (a.K + kw - 1) / kw;
  // The K partition depends on (N, K) only, never on M: every row is then summed in the same order
  // whatever the number of rows in the launch, so a row's result is bit-identical for M = 1..16
  // (the property byteprof's drafting relies on; tests/test_skinny.py:112-121 in the reference).
  const int ref_tiles = (a.N + 31) / 32;
  const int target = 2 * sm_count();
  int S = (target + ref_tiles - 1) / ref_tiles;
  S = S < 1 ? 1 : (S > 8 ? 8 : S);
  if (S > ksteps) S = ksteps;
  const int steps_per_split = (ksteps + S - 1) / S;
  a.k_chunk = steps_per_split * kw;
  S = (a.K + a.k_chunk - 1) / a.k_chunk;

  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(row_tiles, S, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  set_launch_attrs(cfg, attr, S);
  cudaError_t e;
  if (vec)
    e = cudaLaunchKernelEx(&cfg, skinny_fma_kernel<WT, M, R, U, true, XT>, a);
  else
    e = cudaLaunchKernelEx(&cfg, skinny_fma_kernel<WT, M, R, U, false, XT>, a);
  if (e != cudaSuccess)
    return fail(BP_ERR_CUDA, "skinny launch (M=%d N=%d K=%d split=%d): %s", M, a.N, a.K, S, cudaGetErrorString(e));
  return BP_OK;
}

template <typename WT>
int dispatch_m(const SkinnyArgs& a, int m, bool vec, cudaStream_t st) {
  switch (m) {
#define BP_CASE(MM) \
  case MM: return launch_rows<WT, MM, __nv_bfloat16>(a, vec, st);
    BP_CASE(1) BP_CASE(2) BP_CASE(3) BP_CASE(4) BP_CASE(5) BP_CASE(6) BP_CASE(7) BP_CASE(8)
    BP_CASE(9) BP_CASE(10) BP_CASE(11) BP_CASE(12) BP_CASE(13) BP_CASE(14) BP_CASE(15) BP_CASE(16)
#undef BP_CASE
    default: return fail(BP_ERR_INVALID_ARGUMENT, "rows per launch must be 1..16, got %d", m);
  }
}

// fp32 activations: up to 4 rows per launch (the decoder's exactness mode runs one).
constexpr int kF32MaxRows = 4;

template <typename WT>
int dispatch_m_f32(const SkinnyArgs& a, int m, bool vec, cudaStream_t st) {
  switch (m) {
    case 1: return launch_rows<WT, 1, float>(a, vec, st);
    case 2: return launch_rows<WT, 2, float>(a, vec, st);
    case 3: return launch_rows<WT, 3, float>(a, vec, st);
    case 4: return launch_rows<WT, 4, float>(a, vec, st);
    default: return fail(BP_ERR_INVALID_ARGUMENT, "fp32 rows per launch must be 1..%d, got %d", kF32MaxRows, m);
  }
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// BP_SKINNY_PATH (read at every call; for comparisons): "fma" forces the CUDA-core kernels for bf16 and int8,
// "tc" keeps int8 on the tensor cores at every M, "exact" takes the exact int8 CUDA-core kernel wherever it
// applies.
char path_override() {
  const char* e = getenv("BP_SKINNY_PATH");
  return e == nullptr ? 0 : e[0];
}
bool tc_path_enabled() { return path_override() != 'f'; }

// int8 weights go to the exact CUDA-core kernel for one activation row and at most this many output rows
// (only where both exact kernels take the shape, so the choice never changes a bit of the result). Measured,
// graph of a cold weight ring: 2048 x 2048 5.9 us against 6.5 on the tensor cores (two launches: digit prep
// and the main kernel), 2048 x 8192 8.8 against 11.2; the tensor cores win from 8192 rows (8192 x 2048 8.2
// against 12.9) and at M = 4 (2048 x 2048 6.8 against 13.5: dp4a work grows with every row).
constexpr int kI8xMaxN = 4096;

bool use_i8x(const void* x, long long ldx, const void* w, int m, int N, int K) {
  const char o = path_override();
  if (o == 't' || o == 'f') return false;
  if (!skinny_i8x_supported(x, ldx, w, m, N, K) || !skinny_tc_supported(x, ldx, w, m, N, K, true)) return false;
  return o == 'e' || (m == 1 && N <= kI8xMaxN);
}

}  // namespace
}  // namespace bp

extern "C" size_t bp_skinny_workspace_bytes(int M, int N, int K, int w_dtype) {
  if (M <= 0 || N <= 0 || K <= 0) return 0;
  if (w_dtype == BP_DTYPE_INT4) return bp::skinny_i4tc_workspace_bytes(N, K);
  if (w_dtype != BP_DTYPE_BF16 && w_dtype != BP_DTYPE_INT8) return 0;
  return bp::skinny_tc_workspace_bytes(N, K, w_dtype == BP_DTYPE_INT8);
}

extern "C" int bp_device_errors(unsigned int* flags) {
  using namespace bp;
  clear_error();
  if (flags == nullptr) return fail(BP_ERR_INVALID_ARGUMENT, "flags is NULL");
  int st = require_sm100();
  if (st != BP_OK) return st;
  *flags = read_and_clear_device_errors();
  return check_launch("device error read");
}

namespace bp {
namespace {

// The body of bp_skinny_mm: per chunk of up to 16 rows, int8 weights at M <= 4 go to the exact CUDA-core
// kernel (use_i8x), otherwise the tensor-core kernel takes every shape it supports, and the CUDA-core
// streaming kernel the rest.
int skinny_entry(const void* x, long long ldx, const void* w, int w_dtype, const void* w_scale, void* y,
                 long long ldy, int y_dtype, int M, int N, int K, void* workspace, size_t workspace_bytes,
                 void* stream) {
  clear_error();
  if (M < 0 || N < 0 || K < 0) return fail(BP_ERR_INVALID_ARGUMENT, "negative size (M=%d N=%d K=%d)", M, N, K);
  if (w_dtype != BP_DTYPE_BF16 && w_dtype != BP_DTYPE_INT8)
    return fail(BP_ERR_INVALID_ARGUMENT, "weight dtype %d is not bf16 or int8", w_dtype);
  if (y_dtype != BP_DTYPE_BF16 && y_dtype != BP_DTYPE_F32)
    return fail(BP_ERR_INVALID_ARGUMENT, "output dtype %d is not bf16 or fp32", y_dtype);
  if (M == 0 || N == 0) return BP_OK;
  if (y == nullptr) return fail(BP_ERR_INVALID_ARGUMENT, "y is NULL");
  if (ldy < N) return fail(BP_ERR_INVALID_ARGUMENT, "ldy (%lld) < N (%d)", ldy, N);
  int st = require_sm100();
  if (st != BP_OK) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const size_t ysz = y_dtype == BP_DTYPE_F32 ? 4 : 2;
  if (K == 0) {
    cudaError_t e = cudaMemset2DAsync(y, static_cast<size_t>(ldy) * ysz, 0, static_cast<size_t>(N) * ysz, M, s);
    if (e != cudaSuccess) return fail(BP_ERR_CUDA, "zero fill for K = 0: %s", cudaGetErrorString(e));
    return BP_OK;
  }
  if (x == nullptr || w == nullptr) return fail(BP_ERR_INVALID_ARGUMENT, "x or w is NULL");
  if (ldx < K) return fail(BP_ERR_INVALID_ARGUMENT, "ldx (%lld) < K (%d)", ldx, K);
  if (w_dtype == BP_DTYPE_INT8 && w_scale == nullptr)
    return fail(BP_ERR_INVALID_ARGUMENT, "int8 weights need a scale [N]");
  const bool is8 = w_dtype == BP_DTYPE_INT8;
  const int epl = is8 ? 16 : 8;
  const bool vec = aligned16(x) && aligned16(w) && (ldx % 8 == 0) && (K % epl == 0);

  SkinnyArgs a;
  a.ldx = ldx;
  a.w = w;
  a.scale = static_cast<const __nv_bfloat16*>(w_scale);
  a.ldy = ldy;
  a.y_f32 = y_dtype == BP_DTYPE_F32;
  a.N = N;
  a.K = K;
  a.k_chunk = K;
  for (int r0 = 0; r0 < M; r0 += 16) {
    const int m = M - r0 < 16 ? M - r0 : 16;
    a.x = static_cast<const __nv_bfloat16*>(x) + static_cast<long long>(r0) * ldx;
    a.y = static_cast<char*>(y) + static_cast<long long>(r0) * ldy * static_cast<long long>(ysz);
    if (is8 && use_i8x(a.x, ldx, w, m, N, K))
      st = launch_skinny_i8x(a.x, ldx, w, w_scale, a.y, ldy, a.y_f32, m, N, K, s);
    else if (tc_path_enabled() && skinny_tc_supported(a.x, ldx, w, m, N, K, is8))
      st = launch_skinny_tc(a.x, ldx, w, w_scale, a.y, ldy, a.y_f32, m, N, K, is8, workspace, workspace_bytes, s);
    else
      st = is8 ? dispatch_m<int8_t>(a, m, vec, s) : dispatch_m<__nv_bfloat16>(a, m, vec, s);
    if (st != BP_OK) return st;
  }
  return BP_OK;
}

}  // namespace
}  // namespace bp

extern "C" int bp_skinny_mm(const void* x, long long ldx, const void* w, int w_dtype, const void* w_scale, void* y,
                            long long ldy, int y_dtype, int M, int N, int K, void* workspace, size_t workspace_bytes,
                            void* stream) {
  return bp::skinny_entry(x, ldx, w, w_dtype, w_scale, y, ldy, y_dtype, M, N, K, workspace, workspace_bytes, stream);
}

// The int8 GEMV is bp_skinny_mm at M = 1: aligned shapes take one of the two exact kernels (the same bits
// either way), others the CUDA-core kernel.
extern "C" int bp_gemv_int8(const void* x, const int8_t* w, const void* w_scale, void* y, int y_dtype, int N, int K,
                            void* workspace, size_t workspace_bytes, void* stream) {
  return bp::skinny_entry(x, K, w, BP_DTYPE_INT8, w_scale, y, N, y_dtype, 1, N, K, workspace, workspace_bytes, stream);
}

// Skinny linear with fp32 activations on the CUDA-core kernel (the decoder's exactness mode): the same
// weights, K partition and summation order as the bf16-activation kernel, with x read as fp32.
extern "C" int bp_skinny_mm_xf32(const float* x, long long ldx, const void* w, int w_dtype, const void* w_scale,
                                 void* y, long long ldy, int y_dtype, int M, int N, int K, void* stream) {
  using namespace bp;
  clear_error();
  if (M < 0 || N < 0 || K < 0) return fail(BP_ERR_INVALID_ARGUMENT, "negative size (M=%d N=%d K=%d)", M, N, K);
  if (w_dtype != BP_DTYPE_BF16 && w_dtype != BP_DTYPE_INT8)
    return fail(BP_ERR_INVALID_ARGUMENT, "weight dtype %d is not bf16 or int8", w_dtype);
  if (y_dtype != BP_DTYPE_BF16 && y_dtype != BP_DTYPE_F32)
    return fail(BP_ERR_INVALID_ARGUMENT, "output dtype %d is not bf16 or fp32", y_dtype);
  if (M == 0 || N == 0) return BP_OK;
  if (y == nullptr) return fail(BP_ERR_INVALID_ARGUMENT, "y is NULL");
  if (ldy < N) return fail(BP_ERR_INVALID_ARGUMENT, "ldy (%lld) < N (%d)", ldy, N);
  int st = require_sm100();
  if (st != BP_OK) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const size_t ysz = y_dtype == BP_DTYPE_F32 ? 4 : 2;
  if (K == 0) {
    cudaError_t e = cudaMemset2DAsync(y, static_cast<size_t>(ldy) * ysz, 0, static_cast<size_t>(N) * ysz, M, s);
    if (e != cudaSuccess) return fail(BP_ERR_CUDA, "zero fill for K = 0: %s", cudaGetErrorString(e));
    return BP_OK;
  }
  if (x == nullptr || w == nullptr) return fail(BP_ERR_INVALID_ARGUMENT, "x or w is NULL");
  if (ldx < K) return fail(BP_ERR_INVALID_ARGUMENT, "ldx (%lld) < K (%d)", ldx, K);
  if (w_dtype == BP_DTYPE_INT8 && w_scale == nullptr)
    return fail(BP_ERR_INVALID_ARGUMENT, "int8 weights need a scale [N]");
  const bool is8 = w_dtype == BP_DTYPE_INT8;
  const int epl = is8 ? 16 : 8;
  const bool vec = aligned16(x) && aligned16(w) && (ldx % 4 == 0) && (K % epl == 0);
  SkinnyArgs a;
  a.ldx = ldx;
  a.w = w;
  a.scale = static_cast<const __nv_bfloat16*>(w_scale);
  a.ldy = ldy;
  a.y_f32 = y_dtype == BP_DTYPE_F32;
  a.N = N;
  a.K = K;
  a.k_chunk = K;
  for (int r0 = 0; r0 < M; r0 += kF32MaxRows) {
    const int m = M - r0 < kF32MaxRows ? M - r0 : kF32MaxRows;
    a.x = x + static_cast<long long>(r0) * ldx;
    a.y = static_cast<char*>(y) + static_cast<long long>(r0) * ldy * static_cast<long long>(ysz);
    st = is8 ? dispatch_m_f32<int8_t>(a, m, vec, s) : dispatch_m_f32<__nv_bfloat16>(a, m, vec, s);
    if (st != BP_OK) return st;
  }
  return BP_OK;
}
