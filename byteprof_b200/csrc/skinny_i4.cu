// Skinny linear with int4 weights in groups of 128 along K, byteprof's tile-major format, M <= 16 rows per
// launch:  y[m, n] = sum_g scale[g, n] * sum_{k in g} (q[n, k] - zero[g, n]) * x[m, k].
//
// Reference: byteprof/optim/skinny.py:1-19 (the format), 46-63 (_skinny_kernel MODE 3: q - zero rounded to
// bf16 per weight, tl.dot per group, the group scale applied to the fp32 partial) and 136-166 (skinny_mm).
//
// The format: packed uint8 [ceil(N / 32), K / 128, 32, 64]; inside a group of 128 along K, byte j of a row
// holds code j in its low nibble and code j + 64 in its high nibble; the 32 rows of a row tile and one group
// are one contiguous 2 KB block. scale [K / 128, N] bf16, zero [K / 128, N] fp16.
//
// This is the CUDA-core kernel, used below LM-head size (see tc_path_for), without a workspace, for shapes
// the tensor-core kernel does not take (N not a multiple of 8, unaligned scale or zero) and with
// BP_SKINNY_PATH=fma; skinny_i4tc.cu is the tensor-core kernel. Design:
//  * A warp covers 8 rows of a row tile: lane l reads bytes [16 l, 16 l + 16) of the 512-byte slice of
//    each group block, i.e. row l / 4, chunk c = l % 4 (codes 16 c .. 16 c + 15 and 64 + 16 c .. + 15):
//    every load instruction of the warp reads 512 contiguous bytes, streamed with an L2 evict-first policy
//    through a U-deep register pipeline. From M = 2 each lane serves two such row sets (a warp 16 rows),
//    so every staged activation it reads feeds two rows. A CTA covers 64 rows (8 warps, or 4 warps of
//    two rows per lane: half the threads, so two CTAs of ~230 registers a thread fit an SM); split-K
//    over groups forms a thread-block cluster along y whose partials are added through distributed
//    shared memory in rank order (deterministic, no workspace).
//  * A byte b becomes two exact fp32 values: a byte permute gives 0x43bb0000; masking the high nibble
//    away leaves 0x430L0000 = 128 + lo, and the high nibble moved down to bits 16-19 gives 0x430H0000 =
//    128 + hi (the nibble must stay clear of bit 23, the exponent's lowest bit). Per group the lane
//    accumulates P = sum (128 + q) x over its 32 codes, then adds scale * (P - (128 + zero) X) with X the
//    sum of its 32 activations (staged once per CTA): the group term sum (q - zero) x, q - zero exact.
//  * Activations are staged per CTA in shared memory as fp32, four floats of padding per 32 so that the
//    four chunks a warp reads at once fall in different banks.
//  * The K partition depends on (N, K) only, so a row's result does not depend on M.
//  * A row tile past the last one the packed tensor holds (the last CTA of an odd tile count) is never
//    read: those rows read the last tile instead, with scale 0, and are not stored.
#include <cooperative_groups.h>
#include <cuda_fp16.h>
#include <stdlib.h>

#include "bp_common.cuh"
#include "skinny_internal.h"

namespace cg = cooperative_groups;

namespace bp {
namespace {

constexpr int kGroup = 128;
constexpr int kTileRows = 32;
constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kRowsPerCta = 8 * kWarps;
constexpr int kStageBytes = 40 * 1024;  // activation staging budget per CTA
constexpr int kMaxSplit = 8;            // portable cluster size

struct I4Args {
  const __nv_bfloat16* x;
  long long ldx;
  const uint8_t* w;
  const __nv_bfloat16* scale;
  const __half* zero;
  void* y;
  long long ldy;
  int y_f32;
  int N, K, G;
  int g_chunk;  // groups per split
  int gb;       // groups per staging batch (a multiple of the pipeline depth)
};

__device__ __forceinline__ int xs_index(int k) { return k + ((k >> 5) << 2); }
__host__ __device__ constexpr int padded_len(int gb) { return gb * kGroup + (gb * kGroup / 32) * 4; }

__device__ __forceinline__ void store_y(const I4Args& a, int m, int row, float v) {
  if (a.y_f32)
    static_cast<float*>(a.y)[m * a.ldy + row] = v;
  else
    static_cast<__nv_bfloat16*>(a.y)[m * a.ldy + row] = __float2bfloat16_rn(v);
}

// R weight rows per lane: rows warp * 8R + 8r + lane / 4 of the CTA's 64 (r < R; 8 / R warps), so each
// load instruction of a warp still reads 512 contiguous bytes, and every staged activation a lane reads
// from shared memory serves R rows (at R = 2 half the shared-memory reads per FMA). The grid and a row's
// arithmetic (its FMA chains, the lane shuffles, the split order) do not depend on R.
template <int M, int U, int R>
__global__ void __launch_bounds__(kThreads / R) skinny_i4_kernel(const I4Args a) {
  constexpr int kThr = kThreads / R;
  extern __shared__ float xs[];  // [M][padded_len(gb)] activations, then [M][gb][4][2] chunk sums
  __shared__ float part[kRowsPerCta * M];

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int c = lane & 3;
  const int g0 = blockIdx.y * a.g_chunk;
  const int g1 = min(a.G, g0 + a.g_chunk);
  const int plen = padded_len(a.gb);
  float* xsum = xs + M * plen;
  const int ntiles = (a.N + kTileRows - 1) / kTileRows;  // row tiles the packed tensor holds
  pdl_launch_dependents();

  // this lane's 16 bytes of group g of row r: ((t G + g) 32 + rr) 64 + 16 c (padding rows of a tile are
  // zero). A row past the last tile reads the last tile instead (valid memory; its scale is 0 and its
  // result is not stored).
  int row[R];
  bool rv[R];
  const uint8_t* wl[R];
#pragma unroll
  for (int r = 0; r < R; ++r) {
    row[r] = blockIdx.x * kRowsPerCta + warp * 8 * R + 8 * r + (lane >> 2);
    rv[r] = row[r] < a.N;
    const int t = min(row[r] / kTileRows, ntiles - 1), rr = row[r] % kTileRows;
    wl[r] = a.w + (static_cast<long long>(t) * a.G * kTileRows + rr) * 64 + 16 * c;
  }
  const long long gstride = static_cast<long long>(kTileRows) * 64;
  const uint64_t pol = l2_evict_first_policy();

  float acc[R][M];
#pragma unroll
  for (int r = 0; r < R; ++r)
#pragma unroll
    for (int m = 0; m < M; ++m) acc[r][m] = 0.0f;

  uint4 buf[U][R];
  float sc[U][R], zc[U][R];
  auto fetch = [&](int g, int slot_u) {
    // (slot_u is a compile-time index after unrolling)
#pragma unroll
    for (int r = 0; r < R; ++r) {
      if (g < g1) {
        buf[slot_u][r] = ldg_stream16(wl[r] + g * gstride, pol);
        sc[slot_u][r] = rv[r] ? __bfloat162float(a.scale[static_cast<long long>(g) * a.N + row[r]]) : 0.0f;
        zc[slot_u][r] = rv[r] ? __half2float(a.zero[static_cast<long long>(g) * a.N + row[r]]) : 0.0f;
      } else {
        buf[slot_u][r] = make_uint4(0, 0, 0, 0);
        sc[slot_u][r] = zc[slot_u][r] = 0.0f;
      }
    }
  };
#pragma unroll
  for (int u = 0; u < U - 1; ++u) fetch(g0 + u, u);
  pdl_wait_prior_grids();  // the weights above are constants; x may come from the kernel before

  int bb = g0;  // first group of the staged batch
  for (int gg = g0; gg < g1; gg += U) {
    if ((gg - g0) % a.gb == 0) {
      // ---- stage activations of groups [gg, gg + gn) as fp32, then the per-chunk sums ----
      bb = gg;
      const int gn = min(a.gb, g1 - gg);
      __syncthreads();  // the previous batch is consumed
      const int vecs = M * gn * (kGroup / 8);
      for (int i = threadIdx.x; i < vecs; i += kThr) {
        const int m = i / (gn * (kGroup / 8)), kv = (i - m * gn * (kGroup / 8)) * 8;
        const uint4 v = ldg16(a.x + m * a.ldx + static_cast<long long>(gg) * kGroup + kv);
        float* d = xs + m * plen + xs_index(kv);
        *reinterpret_cast<float4*>(d) = make_float4(bf16lo(v.x), bf16hi(v.x), bf16lo(v.y), bf16hi(v.y));
        *reinterpret_cast<float4*>(d + 4) = make_float4(bf16lo(v.z), bf16hi(v.z), bf16lo(v.w), bf16hi(v.w));
      }
      __syncthreads();
      for (int i = threadIdx.x; i < M * gn * 8; i += kThr) {
        const int m = i / (gn * 8), rest = i - m * gn * 8, gl = rest >> 3, cc = (rest >> 1) & 3, h = rest & 1;
        const float* p = xs + m * plen + xs_index(gl * kGroup + 64 * h + 16 * cc);
        float s = 0.0f;
#pragma unroll
        for (int j = 0; j < 16; ++j) s += p[j];
        xsum[((m * a.gb + gl) * 4 + cc) * 2 + h] = s;
      }
      __syncthreads();
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      fetch(gg + u + U - 1, (u + U - 1) % U);  // refill the slot consumed one step ago
      const int g = gg + u;
      if (g < g1) {
        const int gl = g - bb;
        float plo[R][M], phi[R][M];
#pragma unroll
        for (int r = 0; r < R; ++r)
#pragma unroll
          for (int m = 0; m < M; ++m) plo[r][m] = phi[r][m] = 0.0f;
#pragma unroll
        for (int jq = 0; jq < 4; ++jq) {
          float flo[R][4], fhi[R][4];
#pragma unroll
          for (int r = 0; r < R; ++r) {
            const uint32_t word = jq == 0 ? buf[u][r].x : (jq == 1 ? buf[u][r].y : (jq == 2 ? buf[u][r].z : buf[u][r].w));
#pragma unroll
            for (int b = 0; b < 4; ++b) {
              const uint32_t v = __byte_perm(word, 0x43u, 0x4055u | (static_cast<uint32_t>(b) << 8));
              flo[r][b] = __uint_as_float(v & 0xFF0FFFFFu);                            // 128 + low nibble
              fhi[r][b] = __uint_as_float(((v >> 4) & 0x000F0000u) | 0x43000000u);  // 128 + high nibble
            }
          }
#pragma unroll
          for (int m = 0; m < M; ++m) {
            const float4 xl = *reinterpret_cast<const float4*>(xs + m * plen + xs_index(gl * kGroup + 16 * c + 4 * jq));
            const float4 xh =
                *reinterpret_cast<const float4*>(xs + m * plen + xs_index(gl * kGroup + 64 + 16 * c + 4 * jq));
#pragma unroll
            for (int r = 0; r < R; ++r) {
              plo[r][m] = fmaf(flo[r][0], xl.x, plo[r][m]);
              plo[r][m] = fmaf(flo[r][1], xl.y, plo[r][m]);
              plo[r][m] = fmaf(flo[r][2], xl.z, plo[r][m]);
              plo[r][m] = fmaf(flo[r][3], xl.w, plo[r][m]);
              phi[r][m] = fmaf(fhi[r][0], xh.x, phi[r][m]);
              phi[r][m] = fmaf(fhi[r][1], xh.y, phi[r][m]);
              phi[r][m] = fmaf(fhi[r][2], xh.z, phi[r][m]);
              phi[r][m] = fmaf(fhi[r][3], xh.w, phi[r][m]);
            }
          }
        }
#pragma unroll
        for (int r = 0; r < R; ++r) {
          const float cz = 128.0f + zc[u][r];
#pragma unroll
          for (int m = 0; m < M; ++m) {
            const float* sm = xsum + ((m * a.gb + gl) * 4 + c) * 2;
            const float grp = (plo[r][m] + phi[r][m]) - cz * (sm[0] + sm[1]);
            acc[r][m] = fmaf(sc[u][r], grp, acc[r][m]);
          }
        }
      }
    }
  }

  // the row's 4 chunk lanes -> every one of them holds the row sum
#pragma unroll
  for (int r = 0; r < R; ++r)
#pragma unroll
    for (int m = 0; m < M; ++m) {
      acc[r][m] += __shfl_xor_sync(0xffffffffu, acc[r][m], 1);
      acc[r][m] += __shfl_xor_sync(0xffffffffu, acc[r][m], 2);
    }

  if (gridDim.y == 1) {
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
      for (int m = 0; m < M; ++m)
        if ((m & 3) == c && rv[r]) store_y(a, m, row[r], acc[r][m]);
    return;
  }
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const int lr = warp * 8 * R + 8 * r + (lane >> 2);  // row[r] - the CTA's first row
#pragma unroll
    for (int m = 0; m < M; ++m)
      if ((m & 3) == c) part[lr * M + m] = acc[r][m];
  }
  cg::cluster_group cluster = cg::this_cluster();
  cluster.sync();
  const int S = gridDim.y;
  const int rank = static_cast<int>(cluster.block_rank());
  for (int e = rank + S * threadIdx.x; e < kRowsPerCta * M; e += S * kThr) {
    const int rw = blockIdx.x * kRowsPerCta + e / M, m = e % M;
    if (rw >= a.N) continue;
    float s = 0.0f;
    for (int q = 0; q < S; ++q) s += cluster.map_shared_rank(part, q)[e];
    store_y(a, m, rw, s);
  }
  cluster.sync();  // keep this CTA's partials alive until every peer has read them
}

template <int M>
constexpr int pipeline_depth() {
  return M <= 4 ? 4 : (M <= 8 ? 3 : 2);
}

// Rows per lane: two from M = 2, where the shared-memory reads of the staged activations bound the kernel
// (cold L2, 64-row CTAs of 4 warps; M = 16: 2048 x 2048 29.6 -> 13.2 us, 8192 x 2048 65.9 -> 50.9,
// 2048 x 8192 82.8 -> 35.1; M = 4: 6.9 -> 6.4, 16.3 -> 14.7, 16.0 -> 15.1; 128-row CTAs of 8 warps gave
// 23.5 / 49.5 / 63.0 at M = 16, their 8-CTA clusters of full-SM CTAs running in two waves); one at
// M = 1, which is bound by HBM.
template <int M>
constexpr int rows_per_lane() {
  return M >= 2 ? 2 : 1;
}

template <int M>
int launch_i4(I4Args a, cudaStream_t st) {
  constexpr int U = pipeline_depth<M>();
  constexpr int R = rows_per_lane<M>();
  // split from (N, K) only: about two 64-row CTAs per SM in total
  const int row_ctas = (a.N + kRowsPerCta - 1) / kRowsPerCta;
  const int target = 2 * tc_sm_count();
  // rounded down, so that the CTAs fit one wave at two per SM (8192 x 2048, M = 16: 3 splits 51 us, 2 splits
  // 34 us)
  int S = target / row_ctas;
  S = S < 1 ? 1 : (S > kMaxSplit ? kMaxSplit : S);
  if (S > a.G) S = a.G;
  a.g_chunk = (a.G + S - 1) / S;
  S = (a.G + a.g_chunk - 1) / a.g_chunk;
  // staging batch: as many groups as fit the budget, a multiple of U
  const int per_group = M * (padded_len(1) + 8) * static_cast<int>(sizeof(float));
  int gb = kStageBytes / per_group;
  gb = gb < U ? U : gb - gb % U;
  const int chunk_u = (a.g_chunk + U - 1) / U * U;
  if (gb > chunk_u) gb = chunk_u;
  a.gb = gb;
  const size_t smem = static_cast<size_t>(M) * (padded_len(gb) + gb * 8) * sizeof(float);

  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(row_ctas, S, 1);
  cfg.blockDim = dim3(kThreads / R, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  set_launch_attrs(cfg, attr, S);
  const cudaError_t e = cudaLaunchKernelEx(&cfg, skinny_i4_kernel<M, U, R>, a);
  if (e != cudaSuccess)
    return fail(BP_ERR_CUDA, "int4 skinny launch (M=%d N=%d K=%d split=%d): %s", M, a.N, a.K, S, cudaGetErrorString(e));
  return BP_OK;
}

// Which kernel a shape gets. The tensor-core kernel is bound by its MMA rate near 2 TB/s at M <= 4 and
// has a fixed cost of some 10 us per call (the prep kernel and the pipeline fill); the CUDA-core kernel is
// bound by its shared-memory reads of the activations, which grow with M. Measured on the OLMo-2-1B
// shapes: at M = 1 the CUDA-core kernel is 1.5-3x faster below LM-head size and equal on the LM head; at
// M = 16 the tensor-core kernel is 2-4x faster from 8192 x 2048 up. The choice must not depend on M (a
// row's result would then depend on M), so it is by size: tensor cores from 2^26 weights (the LM head),
// which serve the batch-1 decoder as well as the CUDA-core kernel and the verification of many drafted
// positions far better. BP_SKINNY_PATH=fma forces the CUDA-core kernel, BP_SKINNY_PATH=tc the
// tensor-core kernel on every shape it takes (read at every call; for comparisons and tests).
constexpr long long kTcMinWeights = 1LL << 26;
bool tc_path_for(int N, int K) {
  const char* e = getenv("BP_SKINNY_PATH");
  if (e != nullptr && e[0] == 'f') return false;
  if (e != nullptr && e[0] == 't') return true;
  return static_cast<long long>(N) * K >= kTcMinWeights;
}

int dispatch_i4(const I4Args& a, int m, cudaStream_t st) {
  switch (m) {
#define BP_CASE(MM) \
  case MM: return launch_i4<MM>(a, st);
    BP_CASE(1) BP_CASE(2) BP_CASE(3) BP_CASE(4) BP_CASE(5) BP_CASE(6) BP_CASE(7) BP_CASE(8)
    BP_CASE(9) BP_CASE(10) BP_CASE(11) BP_CASE(12) BP_CASE(13) BP_CASE(14) BP_CASE(15) BP_CASE(16)
#undef BP_CASE
    default: return fail(BP_ERR_INVALID_ARGUMENT, "rows per launch must be 1..16, got %d", m);
  }
}

}  // namespace
}  // namespace bp

extern "C" int bp_skinny_mm_int4(const void* x, long long ldx, const uint8_t* w_packed, const void* scale,
                                 const void* zero, void* y, long long ldy, int y_dtype, int M, int N, int K,
                                 int tile_rows, void* workspace, size_t workspace_bytes, void* stream) {
  using namespace bp;
  clear_error();
  if (M < 0 || N < 0 || K < 0) return fail(BP_ERR_INVALID_ARGUMENT, "negative size (M=%d N=%d K=%d)", M, N, K);
  if (y_dtype != BP_DTYPE_BF16 && y_dtype != BP_DTYPE_F32)
    return fail(BP_ERR_INVALID_ARGUMENT, "output dtype %d is not bf16 or fp32", y_dtype);
  if (K % kGroup != 0) return fail(BP_ERR_INVALID_ARGUMENT, "int4 needs K %% 128 == 0 (K=%d)", K);
  if (tile_rows != kTileRows)
    return fail(BP_ERR_UNSUPPORTED, "int4 weights packed with %d rows per tile; the kernel reads 32", tile_rows);
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
  if (x == nullptr || w_packed == nullptr || scale == nullptr || zero == nullptr)
    return fail(BP_ERR_INVALID_ARGUMENT, "x, w, scale or zero is NULL");
  if (ldx < K) return fail(BP_ERR_INVALID_ARGUMENT, "ldx (%lld) < K (%d)", ldx, K);
  if ((reinterpret_cast<uintptr_t>(x) & 15u) != 0 || (reinterpret_cast<uintptr_t>(w_packed) & 15u) != 0 || ldx % 8 != 0)
    return fail(BP_ERR_MISALIGNED, "int4: x and w must be 16-byte aligned and ldx a multiple of 8");

  I4Args a;
  a.ldx = ldx;
  a.w = w_packed;
  a.scale = static_cast<const __nv_bfloat16*>(scale);
  a.zero = static_cast<const __half*>(zero);
  a.ldy = ldy;
  a.y_f32 = y_dtype == BP_DTYPE_F32;
  a.N = N;
  a.K = K;
  a.G = K / kGroup;
  a.g_chunk = a.G;
  a.gb = 1;
  // The tensor-core kernel for every row chunk or for none: the kernel choice depends on the shape, the
  // alignment and the workspace only, so a row's result does not depend on M.
  const bool tc = !(workspace == nullptr && workspace_bytes == 0) && tc_path_for(N, K) &&
                  skinny_i4tc_supported(x, ldx, w_packed, scale, zero, 1, N, K);
  for (int r0 = 0; r0 < M; r0 += 16) {
    const int m = M - r0 < 16 ? M - r0 : 16;
    a.x = static_cast<const __nv_bfloat16*>(x) + static_cast<long long>(r0) * ldx;
    a.y = static_cast<char*>(y) + static_cast<long long>(r0) * ldy * static_cast<long long>(ysz);
    st = tc ? launch_skinny_i4tc(a.x, ldx, w_packed, scale, zero, a.y, ldy, a.y_f32, m, N, K, workspace, workspace_bytes, s)
            : dispatch_i4(a, m, s);
    if (st != BP_OK) return st;
  }
  return BP_OK;
}
