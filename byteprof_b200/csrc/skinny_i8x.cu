// Exact int8 skinny linear on the CUDA cores, for few activation rows (M <= 4):
//   y[m, n] = scale[n] * sum_k q[n, k] x[m, k], with x written exactly as the tensor-core path writes it.
//
// Reference: byteprof/optim/skinny.py:64-75 (_skinny_kernel MODE 1) and byteprof/quant/triton_int8.py:15-47
// (_gemv_int8, the CUDA-core GEMV of one activation row).
//
// Design. The int8 tensor-core kernel (skinny_i8.cu) sums exactly: per activation row m it writes x as the
// fixed-point X = x / 2^(e_m - 29) (e_m the exponent of the row's largest magnitude) in four signed
// base-256 digit planes, forms the exact integer S = sum_k q X and rounds y = fp32(S 2^(e_m - 29) scale)
// once. This kernel forms the same exact S from the same digits with dp4a (four int8 products summed into
// an exact int32 per plane), so its outputs are bit-identical to the tensor-core kernel's: a call may take
// either kernel (here: by M and the weight size) and a row's result still does not depend on the other rows.
//  * One launch, no workspace: every CTA finds the largest |x| of its own K range, the CTAs of a cluster
//    (which cover the whole row) combine them through distributed shared memory into the row exponents, and
//    each CTA writes the digit planes of its K range into shared memory.
//  * Weights stream through a U-deep register pipeline of 16-byte `ld.global.nc.L1::no_allocate` loads
//    with an L2 evict-first policy; a warp covers R weight rows, a lane 16 consecutive bytes of each.
//  * Programmatic dependent launch: the first weight loads are issued before griddepcontrol.wait (weights
//    are not produced by the previous kernel); x is read and y written only after it.
//  * Split-K over a thread-block cluster along grid y: exact int64 partials meet in shared memory and the
//    owner adds them through distributed shared memory (any order gives the same integer).
#include <cooperative_groups.h>

#include "digits.cuh"
#include "skinny_internal.h"
#include "sm100.cuh"

namespace cg = cooperative_groups;

namespace bp {
namespace {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kEPL = 16;           // int8 weights per 16-byte load
constexpr int kKW = 32 * kEPL;     // K covered by one warp step
constexpr int kMaxSplit = 8;       // portable cluster size
constexpr int kMaxRows = 4;        // activation rows per launch

struct I8xArgs {
  const __nv_bfloat16* x;
  long long ldx;
  const int8_t* w;
  const __nv_bfloat16* scale;
  void* y;
  long long ldy;
  int y_f32;
  int N, K;
  int k_chunk;  // K per split, a multiple of kKW
};

__device__ __forceinline__ void store_exact(const I8xArgs& a, int m, int n, long long S, int e) {
  float v;
  if (e == kNonFinite) {
    v = __int_as_float(0x7fffffff);
  } else {  // the tensor-core kernel's rounding: one fp32 rounding of S 2^(e - 29) scale[n], via double
    const double u = __hiloint2double((e - kFracBits + 1023) << 20, 0);  // 2^(e - 29), e >= -127
    v = static_cast<float>(static_cast<double>(S) * u * static_cast<double>(__bfloat162float(a.scale[n])));
  }
  if (a.y_f32)
    static_cast<float*>(a.y)[m * a.ldy + n] = v;
  else
    static_cast<__nv_bfloat16*>(a.y)[m * a.ldy + n] = __float2bfloat16_rn(v);
}

template <int M, int R, int U>
__global__ void __launch_bounds__(kThreads) skinny_i8x_kernel(const I8xArgs a) {
  extern __shared__ __align__(16) uint8_t dig[];  // [M][4 planes][k_chunk] digits of this CTA's K range
  __shared__ long long part[kWarps * R * M];      // this CTA's exact partial sums
  __shared__ uint32_t amax_w[kWarps][M];
  __shared__ uint32_t cta_amax[M];  // read by the cluster's other CTAs
  __shared__ int row_e[M];

  pdl_launch_dependents();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row0 = (blockIdx.x * kWarps + warp) * R;
  const int kb = blockIdx.y * a.k_chunk;
  const int ke = min(a.K, kb + a.k_chunk);
  const int kc = ke - kb;

  bool rv[R];
  const int8_t* wr[R];
#pragma unroll
  for (int r = 0; r < R; ++r) {
    rv[r] = row0 + r < a.N;
    wr[r] = a.w + static_cast<long long>(rv[r] ? row0 + r : 0) * a.K;
  }
  // weights of the first U - 1 steps, requested before the dependency wait
  const uint64_t pol = l2_evict_first_policy();
  uint4 buf[U][R];
  const int k0 = kb + lane * kEPL;
#pragma unroll
  for (int u = 0; u < U - 1; ++u) {
    const int k = k0 + u * kKW;
#pragma unroll
    for (int r = 0; r < R; ++r) buf[u][r] = (rv[r] && k < ke) ? ldg_stream16(wr[r] + k, pol) : make_uint4(0, 0, 0, 0);
  }
  pdl_wait_prior_grids();

  // Row exponents: the largest |x| of this CTA's K range, then over the cluster's CTAs, which together cover
  // the whole row (every CTA gets the same exponent, that of the whole row).
  uint32_t am[M];
#pragma unroll
  for (int m = 0; m < M; ++m) am[m] = 0;
  for (int k = kb + 8 * threadIdx.x; k < ke; k += 8 * kThreads) {
#pragma unroll
    for (int m = 0; m < M; ++m) {
      const uint4 v = ldg16(a.x + m * a.ldx + k);
      const uint32_t wv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int h = 0; h < 4; ++h) am[m] = max(am[m], max(wv[h] & 0x7fffu, (wv[h] >> 16) & 0x7fffu));
    }
  }
#pragma unroll
  for (int m = 0; m < M; ++m) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) am[m] = max(am[m], __shfl_xor_sync(0xffffffffu, am[m], o));
    if (lane == 0) amax_w[warp][m] = am[m];
  }
  __syncthreads();
  if (threadIdx.x < M) {
    uint32_t mx = 0;
    for (int w = 0; w < kWarps; ++w) mx = max(mx, amax_w[w][threadIdx.x]);
    cta_amax[threadIdx.x] = mx;
  }
  cg::cluster_group cluster = cg::this_cluster();
  const int S = gridDim.y;
  if (S > 1) cluster.sync();  // every CTA's maxima written
  else __syncthreads();
  if (threadIdx.x < M) {
    uint32_t mx = 0;
    for (int q = 0; q < S; ++q) mx = max(mx, S > 1 ? cluster.map_shared_rank(cta_amax, q)[threadIdx.x] : cta_amax[threadIdx.x]);
    row_e[threadIdx.x] = row_exponent(mx);
  }
  __syncthreads();
  // digit planes of this CTA's K range (a row holding Inf or NaN: zero digits, NaN output)
  for (int j = threadIdx.x; j < M * (kc / 8); j += kThreads) {
    const int m = j / (kc / 8), c = (j - m * (kc / 8)) * 8;
    const int e = row_e[m];
    uint4 v = ldg16(a.x + m * a.ldx + kb + c);
    if (e == kNonFinite) v = make_uint4(0, 0, 0, 0);
    uint32_t pl[kDigitPlanes][2];
    digitise8(v, e == kNonFinite ? 0 : e, pl);
#pragma unroll
    for (int p = 0; p < kDigitPlanes; ++p)
      *reinterpret_cast<uint2*>(dig + (static_cast<size_t>(m) * kDigitPlanes + p) * a.k_chunk + c) =
          make_uint2(pl[p][0], pl[p][1]);
  }
  __syncthreads();

  int acc[R][M][kDigitPlanes];
#pragma unroll
  for (int r = 0; r < R; ++r)
#pragma unroll
    for (int m = 0; m < M; ++m)
#pragma unroll
      for (int p = 0; p < kDigitPlanes; ++p) acc[r][m][p] = 0;

  for (int kk = k0; kk < ke; kk += U * kKW) {
#pragma unroll
    for (int u = 0; u < U; ++u) {
      {  // refill the slot consumed one step ago with the step U - 1 ahead
        const int kn = kk + (u + U - 1) * kKW;
#pragma unroll
        for (int r = 0; r < R; ++r)
          buf[(u + U - 1) % U][r] = (rv[r] && kn < ke) ? ldg_stream16(wr[r] + kn, pol) : make_uint4(0, 0, 0, 0);
      }
      const int k = kk + u * kKW;
      if (k < ke) {
        uint4 d[M][kDigitPlanes];
#pragma unroll
        for (int m = 0; m < M; ++m)
#pragma unroll
          for (int p = 0; p < kDigitPlanes; ++p)
            d[m][p] = *reinterpret_cast<const uint4*>(dig + (static_cast<size_t>(m) * kDigitPlanes + p) * a.k_chunk +
                                                      (k - kb));
#pragma unroll
        for (int r = 0; r < R; ++r) {
          const uint4 q = buf[u][r];
#pragma unroll
          for (int m = 0; m < M; ++m)
#pragma unroll
            for (int p = 0; p < kDigitPlanes; ++p) {
              int s = acc[r][m][p];
              s = __dp4a(static_cast<int>(q.x), static_cast<int>(d[m][p].x), s);
              s = __dp4a(static_cast<int>(q.y), static_cast<int>(d[m][p].y), s);
              s = __dp4a(static_cast<int>(q.z), static_cast<int>(d[m][p].z), s);
              s = __dp4a(static_cast<int>(q.w), static_cast<int>(d[m][p].w), s);
              acc[r][m][p] = s;
            }
        }
      }
    }
  }

  // exact sums: planes combined in int64, then over the warp's lanes
  long long tot[R][M];
#pragma unroll
  for (int r = 0; r < R; ++r)
#pragma unroll
    for (int m = 0; m < M; ++m) {
      long long v = static_cast<long long>(acc[r][m][0]) + (static_cast<long long>(acc[r][m][1]) << 8) +
                    (static_cast<long long>(acc[r][m][2]) << 16) + (static_cast<long long>(acc[r][m][3]) << 24);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
      tot[r][m] = v;
    }

  if (gridDim.y == 1) {
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
      for (int m = 0; m < M; ++m)
        if (((r * M + m) & 31) == lane && rv[r]) store_exact(a, m, row0 + r, tot[r][m], row_e[m]);
    return;
  }

  // split-K: rank s of the cluster holds the partial of split s; the owner of each output adds them
  if (lane == 0) {
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
      for (int m = 0; m < M; ++m) part[(warp * R + r) * M + m] = tot[r][m];
  }
  cluster.sync();
  const int rank = static_cast<int>(cluster.block_rank());
  const int tile_row0 = blockIdx.x * kWarps * R;
  for (int e = rank + S * threadIdx.x; e < kWarps * R * M; e += S * kThreads) {
    const int rr = e / M, m = e - rr * M;
    const int row = tile_row0 + rr;
    if (row >= a.N) continue;
    long long s = 0;
    for (int q = 0; q < S; ++q) s += cluster.map_shared_rank(part, q)[e];
    store_exact(a, m, row, s, row_e[m]);
  }
  cluster.sync();  // keep this CTA's partials alive until every peer has read them
}

template <int M>
struct I8xTile {  // weight rows per warp and pipeline depth
  static constexpr int R = M <= 2 ? 4 : 2;
  static constexpr int U = 3;
};

int sms() {
  static int cached[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return 148;
  if (cached[dev] == 0) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    cached[dev] = n > 0 ? n : 148;
  }
  return cached[dev];
}

// K per split: two CTAs per SM over the row tiles of 32 rows (the same rule for every M), whole warp steps.
int split_chunk(int N, int K) {
  const int ref_tiles = (N + 31) / 32;
  int S = (2 * sms() + ref_tiles - 1) / ref_tiles;
  S = S < 1 ? 1 : (S > kMaxSplit ? kMaxSplit : S);
  const int ksteps = (K + kKW - 1) / kKW;
  if (S > ksteps) S = ksteps;
  return ((ksteps + S - 1) / S) * kKW;
}

size_t digit_bytes(int M, int N, int K) { return static_cast<size_t>(M) * kDigitPlanes * split_chunk(N, K); }

template <int M>
int launch_i8x(I8xArgs a, cudaStream_t st) {
  constexpr int R = I8xTile<M>::R, U = I8xTile<M>::U;
  a.k_chunk = split_chunk(a.N, a.K);
  const int S = (a.K + a.k_chunk - 1) / a.k_chunk;
  const size_t smem = digit_bytes(M, a.N, a.K);
  static bool attr_done[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr_done[dev]) {
    const cudaError_t e = cudaFuncSetAttribute(skinny_i8x_kernel<M, R, U>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               static_cast<int>(kI8xMaxDigitBytes));
    if (e != cudaSuccess) return fail(BP_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
    attr_done[dev] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((a.N + kWarps * R - 1) / (kWarps * R), S, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  int na = 0;
  if (tc_pdl_enabled()) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  if (S > 1) {
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = 1;
    attr[na].val.clusterDim.y = S;
    attr[na].val.clusterDim.z = 1;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, skinny_i8x_kernel<M, R, U>, a);
  if (e != cudaSuccess)
    return fail(BP_ERR_CUDA, "exact int8 skinny launch (M=%d N=%d K=%d split=%d): %s", M, a.N, a.K, S,
                cudaGetErrorString(e));
  return BP_OK;
}

}  // namespace

bool skinny_i8x_supported(const void* x, long long ldx, const void* w, int M, int N, int K) {
  const bool al = (reinterpret_cast<uintptr_t>(x) & 15u) == 0 && (reinterpret_cast<uintptr_t>(w) & 15u) == 0;
  return al && M >= 1 && M <= kMaxRows && N >= 1 && K >= 16 && K % 16 == 0 && K <= 131072 && ldx % 8 == 0 &&
         digit_bytes(M, N, K) <= kI8xMaxDigitBytes;
}

int launch_skinny_i8x(const void* x, long long ldx, const void* w, const void* w_scale, void* y, long long ldy, int y_f32,
                      int M, int N, int K, cudaStream_t stream) {
  I8xArgs a;
  a.x = static_cast<const __nv_bfloat16*>(x);
  a.ldx = ldx;
  a.w = static_cast<const int8_t*>(w);
  a.scale = static_cast<const __nv_bfloat16*>(w_scale);
  a.y = y;
  a.ldy = ldy;
  a.y_f32 = y_f32;
  a.N = N;
  a.K = K;
  a.k_chunk = K;
  switch (M) {
    case 1: return launch_i8x<1>(a, stream);
    case 2: return launch_i8x<2>(a, stream);
    case 3: return launch_i8x<3>(a, stream);
    case 4: return launch_i8x<4>(a, stream);
    default: return fail(BP_ERR_INVALID_ARGUMENT, "exact int8 CUDA-core kernel takes 1..%d rows, got %d", kMaxRows, M);
  }
}

}  // namespace bp
