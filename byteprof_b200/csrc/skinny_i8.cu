// Tensor-core skinny linear with int8 weights and a per-row bf16 scale, M <= 16 activation rows per launch:
//   y[m, n] = scale[n] * sum_k q[n, k] x[m, k].
//
// Reference: byteprof/optim/skinny.py:35-80 (_skinny_kernel MODE 1: the int8 tile widened to bf16 before
// tl.dot, fp32 accumulation, the per-row scale applied to the accumulator) and byteprof/quant/int8.py
// (the int8 GEMV for M = 1); the result is cast to the output dtype once, from fp32.
//
// B200 design. A tcgen05 MMA costs about the same whatever its N (up to 128; 256 costs less than twice),
// so the weights must be the MMA's wide operand: B = the int8 weight tile (N = 128 or 256 rows), fed by TMA
// straight from HBM to shared memory with no widening pass. The integer MMA (kind::i8) needs an int8 A,
// so the bf16 activations are written exactly as fixed-point numbers of four signed base-256 digits:
//  * per activation row m, e_m = exponent of max_k |x[m, k]| and x = X 2^(e_m - 29) with |X| < 2^30;
//    bf16 values down to 2^-22 of the row maximum are exact, smaller ones are rounded to the nearest
//    multiple of 2^(e_m - 29) (an error below 2^-29 of the row maximum);
//  * X = d0 + 2^8 d1 + 2^16 d2 + 2^24 d3 with d_p in [-128, 127]; row 4 m + p of the digit matrix holds
//    plane d_p of row m, and a 64-row A tile (MMA M = 64) gives all four planes of all 16 rows in one MMA.
//    A small kernel per call computes the exponents and the [4 M, K] digit matrix into the workspace
//    (once, instead of once per weight tile), overlapped with the main kernel's first weight loads;
//  * int32 accumulation is exact (|sum| <= 128 * 128 * K < 2^31 for K <= 131072); the planes are combined
//    exactly in int64 as S = D0 + 2^8 D1 + 2^16 D2 + 2^24 D3 and y = fp32(S * 2^(e_m - 29) * scale[n]),
//    so y is the correctly rounded value of the exact sum over the fixed-point activations, and partial
//    sums of a split K range add exactly: the result does not depend on how K was split.
//  * Two partitions, chosen from (N, K) only: stream-K over (256-row tile, 128-wide k-block) units on a
//    persistent grid of one CTA per SM, split tiles finished by the CTA that arrives last (exact int64
//    partials in the workspace); or, for few tiles, 128-row tiles whose K range is split over the S CTAs
//    of a cluster; each CTA stores its exact sums of every column into a slot of the CTA owning that
//    column (distributed shared memory), and after one cluster barrier the owner adds its S slots.
//  * TMEM: two accumulators of TN int32 columns, so draining one tile overlaps the next tile's MMAs. For
//    M = 64 the MMA writes D row i to TMEM lane 32 (i / 16) + i % 16: the four planes of activation rows
//    4 q .. 4 q + 3 sit in lanes 0-15 of quadrant q; each epilogue warp moves a 32-column chunk of them
//    through shared memory so that every lane combines and stores 4 (row, column) outputs.
//  * Warp roles: 0 weight TMA, 1 MMA issue + TMEM owner, 2 digit-tile TMA (64 x 128 bytes, rows beyond
//    4 M zero-filled), 3-6 epilogue.
//  * Programmatic dependent launch: weights are requested before griddepcontrol.wait; the exponents and
//    digits are read and y is written only after it.
//  * Every mbarrier wait is bounded; a timeout sets the device error word, the CTA drains its copies in
//    flight, frees TMEM and returns.
#include <cudaTypedefs.h>

#include "digits.cuh"
#include "skinny_internal.h"
#include "sm100.cuh"

namespace bp {
namespace {

constexpr int kBK = 128;                   // K per unit: one 128-byte swizzle row of int8
constexpr int kRows = 16;                  // activation rows per launch
constexpr int kPlanes = kDigitPlanes;      // base-256 digits per activation
constexpr int kAM = kRows * kPlanes;       // MMA M
constexpr int kABytes = kAM * kBK;         // 8 KB
constexpr int kThreads = 224;              // weight TMA, MMA, digit TMA, 4 epilogue warps
constexpr int kEpiWarp0 = 3;
constexpr int kGroup = 128;                // epilogue threads
constexpr int kMaxClusterSplit = 8;        // portable cluster size
constexpr size_t kExpBytes = 1024;         // workspace: row exponents after the tile counters, then the digits
constexpr int kL2Ahead = 7;                // units requested into L2 beyond the weight ring at the start

// TN = 256: stream-K, one CTA per SM with 160 KB of weights in flight. TN = 128: cluster split-K, where a
// CTA streams only a few units: a shorter ring, so that two CTAs fit per SM and the next call's CTAs start
// (and request their weights) under this call's tail.
template <int TN>
struct I8Cfg {
  static constexpr int kWStages = TN == 256 ? 5 : 4;
  static constexpr int kAStages = TN == 256 ? 6 : 2;
  static constexpr int kMinBlocks = TN == 256 ? 1 : 2;
  static constexpr int kWBytes = TN * kBK;
  // cluster mode: [source rank][row][column of the owner's share] exact partials (S * R <= TN + S - 1)
  static constexpr int kRedElems = TN == 128 ? kRows * (TN + kMaxClusterSplit) : 2;
  static constexpr uint32_t kTmemCols = 2 * TN;
};

struct I8Args {
  void* y;
  long long ldy;
  int y_f32;
  const __nv_bfloat16* scale;
  const int* exps;       // [M] row exponents (workspace)
  int M, N, K;
  int tiles, kblocks;
  long long units;
  int P;
  int S;                 // cluster mode: CTAs per tile
  int* counters;         // stream-K: [tiles], zero between launches
  long long* partials;   // stream-K: [P][2][kRows][TN]
};

template <int TN>
struct __align__(1024) I8Smem {
  uint8_t w[I8Cfg<TN>::kWStages][I8Cfg<TN>::kWBytes];
  uint8_t a[I8Cfg<TN>::kAStages][kABytes];
  long long red[I8Cfg<TN>::kRedElems];  // cluster mode: the peers' exact partials of this CTA's columns
  uint64_t full[I8Cfg<TN>::kWStages], empty[I8Cfg<TN>::kWStages];
  uint64_t afull[I8Cfg<TN>::kAStages], aempty[I8Cfg<TN>::kAStages];
  uint64_t tfull[2], tempty[2];
  uint64_t mma_done;
  float tscale[TN];
  uint4 xpose[4][16][8];  // per epilogue warp: 16 TMEM lanes x 32 int32 columns, for the plane transpose
  int row_exp[kRows];
  uint32_t tmem_base;
  int abort;
  int last_flag;
};
template <int TN>
constexpr size_t smem_bytes() {
  return sizeof(I8Smem<TN>) + 1024;
}
static_assert(smem_bytes<256>() <= 232448, "shared memory per CTA");
static_assert(smem_bytes<128>() <= 115712, "two CTAs per SM (228 KB, 1 KB reserved per CTA)");

__device__ __forceinline__ long long unit_start(int c, long long U, int P) { return static_cast<long long>(c) * U / P; }
__device__ __forceinline__ int unit_owner(long long u, long long U, int P) {
  return static_cast<int>(((u + 1) * P - 1) / U);
}

__device__ __forceinline__ void wait_drain(uint64_t* bar, uint32_t parity) {
  const unsigned long long t0 = globaltimer();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer() - t0 > kWaitLimitNs) {
      atomicOr(&g_bp_device_errors, BP_DEVERR_TIMEOUT);
      return;
    }
  }
}

__device__ __forceinline__ void store_i8(const I8Args& a, int m, int n, long long S, int e, float scale) {
  float v;
  if (e == kNonFinite) {
    v = __int_as_float(0x7fffffff);
  } else {
    const double u = __hiloint2double((e - kFracBits + 1023) << 20, 0);  // 2^(e - 29), e >= -127
    v = static_cast<float>(static_cast<double>(S) * u * static_cast<double>(scale));
  }
  if (a.y_f32)
    static_cast<float*>(a.y)[m * a.ldy + n] = v;
  else
    static_cast<__nv_bfloat16*>(a.y)[m * a.ldy + n] = __float2bfloat16_rn(v);
}

// Row exponents and the [4 M, K] digit matrix (row 4 m + p: plane p of activation row m) of the M
// activation rows, one CTA per row, for the main kernel that follows.
__global__ void __launch_bounds__(256) i8_digitise_kernel(const __nv_bfloat16* x, long long ldx, int K, int* exps,
                                                          uint8_t* digits) {
  pdl_launch_dependents();  // the main kernel may start streaming weights now
  pdl_wait_prior_grids();   // x may come from the previous kernel
  const int m = blockIdx.x;
  const __nv_bfloat16* xr = x + static_cast<long long>(m) * ldx;
  // the first 8192 values of the row stay in registers for the digit pass (one read of x for K <= 8192)
  uint32_t amax = 0;
  uint4 keep[4];
  for (int k0 = 8 * threadIdx.x; k0 < K; k0 += 4 * 8 * 256) {
    uint4 v[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int k = k0 + j * 8 * 256;
      v[j] = k < K ? __ldcg(reinterpret_cast<const uint4*>(xr + k)) : make_uint4(0, 0, 0, 0);
    }
    if (k0 == 8 * static_cast<int>(threadIdx.x))
#pragma unroll
      for (int j = 0; j < 4; ++j) keep[j] = v[j];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t wv[4] = {v[j].x, v[j].y, v[j].z, v[j].w};
#pragma unroll
      for (int h = 0; h < 4; ++h) amax = max(amax, max(wv[h] & 0x7fffu, (wv[h] >> 16) & 0x7fffu));
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = max(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  __shared__ uint32_t red[8];
  __shared__ int e_row;
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
  __syncthreads();
  if (threadIdx.x == 0) {
    uint32_t mx = 0;
    for (int w = 0; w < 8; ++w) mx = max(mx, red[w]);
    e_row = row_exponent(mx);
    exps[m] = e_row;
  }
  __syncthreads();
  const bool nonfinite = e_row == kNonFinite;  // the row's output is NaN; its digits are zero
  const int e = nonfinite ? 0 : e_row;
  uint8_t* drow = digits + static_cast<size_t>(4 * m) * K;
  for (int k0 = 8 * threadIdx.x; k0 < K; k0 += 4 * 8 * 256) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int k = k0 + j * 8 * 256;
      if (k >= K) break;
      uint4 v = k0 == 8 * static_cast<int>(threadIdx.x) ? keep[j] : __ldcg(reinterpret_cast<const uint4*>(xr + k));
      if (nonfinite) v = make_uint4(0, 0, 0, 0);
      uint32_t pl[kPlanes][2];
      digitise8(v, e, pl);
#pragma unroll
      for (int p = 0; p < kPlanes; ++p)
        *reinterpret_cast<uint2*>(drow + static_cast<size_t>(p) * K + k) = make_uint2(pl[p][0], pl[p][1]);
    }
  }
}

// kCluster = false: stream-K over (tile, k-block) units, split tiles finished through the workspace.
// kCluster = true: grid = tiles x S, the S CTAs of a cluster split one tile's K range and add their exact
// partials through distributed shared memory, in rank order.
template <int TN, bool kCluster>
__global__ void __launch_bounds__(kThreads, I8Cfg<TN>::kMinBlocks)
    skinny_i8_kernel(const __grid_constant__ CUtensorMap tw, const __grid_constant__ CUtensorMap ta, const I8Args a) {
  using Cfg = I8Cfg<TN>;
  constexpr int kWStages = Cfg::kWStages, kAStages = Cfg::kAStages;
  extern __shared__ uint8_t smem_raw[];
  I8Smem<TN>& s =
      *reinterpret_cast<I8Smem<TN>*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int c = blockIdx.x;
  const long long U = a.units;
  const int KB = a.kblocks;
  long long u0, u1;
  int rank = 0;
  if constexpr (kCluster) {
    rank = static_cast<int>(cluster_ctarank());
    const long long t = cluster_id_x();
    u0 = t * KB + static_cast<long long>(rank) * KB / a.S;
    u1 = t * KB + static_cast<long long>(rank + 1) * KB / a.S;
  } else {
    u0 = unit_start(c, U, a.P);
    u1 = unit_start(c + 1, U, a.P);
  }
  const int n_units = static_cast<int>(u1 - u0);
  const int t_first = static_cast<int>(u0 / KB);
  const int t_last = n_units > 0 ? static_cast<int>((u1 - 1) / KB) : t_first - 1;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kWStages; ++i) {
      mbar_init(&s.full[i], 1);
      mbar_init(&s.empty[i], 1);
    }
    for (int i = 0; i < kAStages; ++i) {
      mbar_init(&s.afull[i], 1);
      mbar_init(&s.aempty[i], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&s.tfull[b], 1);
      mbar_init(&s.tempty[b], kGroup);
    }
    mbar_init(&s.mma_done, 1);
    s.abort = 0;
    s.last_flag = 0;
    mbar_fence_init();
    tma_prefetch_desc(&tw);
    tma_prefetch_desc(&ta);
  }
  if (warp == 1) {
    tmem_alloc(&s.tmem_base, Cfg::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before_sync();
  __syncthreads();
  tc_fence_after_sync();
  pdl_launch_dependents();
  const uint32_t tmem = s.tmem_base;
  volatile int* abort = &s.abort;

  if (warp == 0) {
    if (lane == 0) {
      // ---- weight tiles: TMA, no dependence on the previous kernels ----
      const uint64_t pol = l2_evict_first_policy();
      int issued = 0;
      for (int i = 0; i < n_units; ++i) {
        const int st = i % kWStages;
        if (i >= kWStages && !mbar_wait(&s.empty[st], static_cast<uint32_t>((i / kWStages) + 1) & 1u, abort)) break;
        const long long u = u0 + i;
        const int t = static_cast<int>(u / KB), kb = static_cast<int>(u % KB);
        mbar_arrive_expect_tx(&s.full[st], Cfg::kWBytes);
        tma_load_2d_hint(s.w[st], &tw, &s.full[st], kb * kBK, t * TN, pol);
        issued = i + 1;
        if (i == kWStages - 1) {
          // The ring is full before the digits (the prep kernel's output) can arrive: request the next units
          // into L2, so that the ring refills from L2 once the MMAs start.
          for (int j = kWStages; j < n_units && j < kWStages + kL2Ahead; ++j) {
            const long long uj = u0 + j;
            tma_prefetch_l2_2d(&tw, static_cast<int>(uj % KB) * kBK, static_cast<int>(uj / KB) * TN);
          }
        }
      }
      for (int st = 0; st < kWStages && st < issued; ++st) {  // drain
        const int i_last = st + kWStages * ((issued - 1 - st) / kWStages);
        wait_drain(&s.full[st], static_cast<uint32_t>(i_last / kWStages) & 1u);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---- MMA issuer: 4 x (M 64, N TN, K 32) per unit ----
      constexpr uint32_t idesc = umma_idesc_s8(kAM, TN);
      int i = 0, it = 0;
      bool ok = true;
      for (int t = t_first; t <= t_last && ok; ++t, ++it) {
        const long long lo = u0 > static_cast<long long>(t) * KB ? u0 : static_cast<long long>(t) * KB;
        const long long hi = u1 < static_cast<long long>(t + 1) * KB ? u1 : static_cast<long long>(t + 1) * KB;
        const int buf = it & 1;
        if (!mbar_wait(&s.tempty[buf], static_cast<uint32_t>((it >> 1) + 1) & 1u, abort)) break;
        tc_fence_after_sync();
        const uint32_t dacc = tmem + static_cast<uint32_t>(buf * TN);
        for (long long u = lo; u < hi; ++u, ++i) {
          const int ws = i % kWStages, as = i % kAStages;
          if (!mbar_wait(&s.full[ws], static_cast<uint32_t>(i / kWStages) & 1u, abort) ||
              !mbar_wait(&s.afull[as], static_cast<uint32_t>(i / kAStages) & 1u, abort)) {
            ok = false;
            break;
          }
          tc_fence_after_sync();
          const uint32_t ab = smem_addr(s.a[as]), wb = smem_addr(s.w[ws]);
#pragma unroll
          for (int kk = 0; kk < kBK / 32; ++kk)
            umma_i8(dacc, umma_desc_sw128(ab + 32 * kk), umma_desc_sw128(wb + 32 * kk), idesc,
                    (u > lo || kk > 0) ? 1u : 0u);
          umma_commit(&s.empty[ws]);   // the weight stage is free once these MMAs have read it
          umma_commit(&s.aempty[as]);  // and so is the digit tile
        }
        if (ok) umma_commit(&s.tfull[buf]);
      }
      umma_commit(&s.mma_done);
      wait_drain(&s.mma_done, 0);
    }
  } else if (warp == 2) {
    if (lane == 0) {
      // ---- digit tiles: TMA from the digit matrix the previous kernel wrote ----
      pdl_wait_prior_grids();
      int issued = 0;
      for (int i = 0; i < n_units; ++i) {
        const int as = i % kAStages;
        if (i >= kAStages && !mbar_wait(&s.aempty[as], static_cast<uint32_t>((i / kAStages) + 1) & 1u, abort)) break;
        const int kb = static_cast<int>((u0 + i) % KB);
        mbar_arrive_expect_tx(&s.afull[as], kABytes);
        tma_load_2d(s.a[as], &ta, &s.afull[as], kb * kBK, 0);
        issued = i + 1;
      }
      for (int as = 0; as < kAStages && as < issued; ++as) {  // drain
        const int i_last = as + kAStages * ((issued - 1 - as) / kAStages);
        wait_drain(&s.afull[as], static_cast<uint32_t>(i_last / kAStages) & 1u);
      }
    }
  } else {
    // ---- epilogue ----
    pdl_wait_prior_grids();
    const int et = threadIdx.x - 32 * kEpiWarp0;
    if (et < kRows) s.row_exp[et] = et < a.M ? __ldcg(a.exps + et) : 0;
    named_barrier_sync(1, kGroup);
    const int q = warp & 3;               // TMEM lane quadrant: activation rows 4 q .. 4 q + 3
    const int g = lane >> 3;              // this lane finishes row m = 4 q + g, columns 4 (lane % 8) .. + 3
    const int m = 4 * q + g;              // of each 32-column chunk
    const int cl = 4 * (lane & 7);
    const bool writer = m < a.M;
    const int e = s.row_exp[m];
    uint4 (&xp)[16][8] = s.xpose[q];
    int it = 0;
    for (int t = t_first; t <= t_last; ++t, ++it) {
      const int buf = it & 1;
      float sc[TN / kGroup];  // this tile's scales, staged through shared memory
#pragma unroll
      for (int h = 0; h < TN / kGroup; ++h) {
        const int n = t * TN + et + kGroup * h;
        sc[h] = n < a.N ? __bfloat162float(a.scale[n]) : 0.0f;
      }
      const bool ok = mbar_wait(&s.tfull[buf], static_cast<uint32_t>(it >> 1) & 1u, abort);
      __syncwarp();
      if (named_barrier_or(1, kGroup, !ok)) break;  // (also: every thread is done with the previous scales)
#pragma unroll
      for (int h = 0; h < TN / kGroup; ++h) s.tscale[et + kGroup * h] = sc[h];
      named_barrier_sync(1, kGroup);
      tc_fence_after_sync();
      bool owned = true;
      long long* mine = nullptr;
      int c_lo = c, c_hi = c;
      if constexpr (!kCluster) {
        c_lo = unit_owner(static_cast<long long>(t) * KB, U, a.P);
        c_hi = unit_owner(static_cast<long long>(t + 1) * KB - 1, U, a.P);
        owned = c_lo == c_hi;
        mine = a.partials + (static_cast<size_t>(c * 2 + (t == t_first ? 0 : 1)) * kRows + m) * TN;
      }
      const int R = kCluster ? (TN + a.S - 1) / a.S : TN;  // cluster mode: rank c / R owns column c
      const int slot0 = kCluster ? static_cast<int>(rank) * kRows * R : 0;  // this CTA's slot in each owner
#pragma unroll 1
      for (int ch = 0; ch < TN / 32; ++ch) {
        uint32_t raw[32];
        tmem_ld_32x32b_x32(tmem + (static_cast<uint32_t>(32 * q) << 16) + static_cast<uint32_t>(buf * TN + 32 * ch), raw);
        __syncwarp();  // the previous chunk's reads of xp are done
        if (lane < 16) {
#pragma unroll
          for (int j = 0; j < 8; ++j)  // 16-byte chunk j of row `lane`, rotated by the row to spread banks
            xp[lane][(j + lane) & 7] = make_uint4(raw[4 * j], raw[4 * j + 1], raw[4 * j + 2], raw[4 * j + 3]);
        }
        __syncwarp();
        if (writer) {
          // planes 0-3 of row m are TMEM lanes 4 g + p; exact S = D0 + 2^8 D1 + 2^16 D2 + 2^24 D3
          long long v[4];
          {
            uint4 d[4];
#pragma unroll
            for (int p = 0; p < 4; ++p) d[p] = xp[4 * g + p][((cl >> 2) + 4 * g + p) & 7];
            const int d0[4] = {int(d[0].x), int(d[0].y), int(d[0].z), int(d[0].w)};
            const int d1[4] = {int(d[1].x), int(d[1].y), int(d[1].z), int(d[1].w)};
            const int d2[4] = {int(d[2].x), int(d[2].y), int(d[2].z), int(d[2].w)};
            const int d3[4] = {int(d[3].x), int(d[3].y), int(d[3].z), int(d[3].w)};
#pragma unroll
            for (int i = 0; i < 4; ++i)
              v[i] = static_cast<long long>(d0[i]) + 256LL * d1[i] + 65536LL * d2[i] + 16777216LL * d3[i];
          }
          const int c0 = 32 * ch + cl;
          if constexpr (kCluster) {
            // this CTA's exact partial goes to the owning CTA's slot for this rank (remote stores)
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const int col = c0 + i, own = col / R;
              const uint32_t dst =
                  mapa_shared(smem_addr(&s.red[slot0 + m * R + (col - own * R)]), static_cast<uint32_t>(own));
              asm volatile("st.shared::cluster.u64 [%0], %1;" ::"r"(dst), "l"(v[i]) : "memory");
            }
          } else if (owned) {
            const int n0 = t * TN + c0;
#pragma unroll
            for (int i = 0; i < 4; ++i)
              if (n0 + i < a.N) store_i8(a, m, n0 + i, v[i], e, s.tscale[c0 + i]);
          } else {
            *reinterpret_cast<longlong2*>(mine + c0) = make_longlong2(v[0], v[1]);
            *reinterpret_cast<longlong2*>(mine + c0 + 2) = make_longlong2(v[2], v[3]);
          }
        }
      }
      tc_fence_before_sync();
      mbar_arrive(&s.tempty[buf]);
      if (kCluster || owned) continue;
      __syncwarp();
      named_barrier_sync(1, kGroup);  // every partial of this CTA is written ...
      if (et == 0) {
        __threadfence();  // ... and (cumulatively) visible GPU-wide before the arrival is counted
        const int old = atomicAdd(&a.counters[t], 1);
        const int last = old == c_hi - c_lo;
        if (last) {
          a.counters[t] = 0;  // every contributor has arrived: ready for the next launch
          __threadfence();
        }
        s.last_flag = last;
      }
      __syncwarp();
      named_barrier_sync(1, kGroup);
      if (s.last_flag) {
        // exact int64 sums of the contributors' partials: pairs of columns (16-byte loads), four pairs and
        // up to four contributors in flight per thread
        const int npairs = a.M * (TN / 2);
        for (int p0 = et; p0 < npairs; p0 += 4 * kGroup) {
          longlong2 acc[4];
#pragma unroll
          for (int j = 0; j < 4; ++j) acc[j] = make_longlong2(0, 0);
          for (int cc0 = c_lo; cc0 <= c_hi; cc0 += 4) {
            longlong2 v[4][4];
#pragma unroll
            for (int g = 0; g < 4; ++g) {
              const int cc = cc0 + g;
              const int cs = cc <= c_hi && t != static_cast<int>(unit_start(cc, U, a.P) / KB) ? 1 : 0;
              const long long* base = a.partials + static_cast<size_t>(cc * 2 + cs) * kRows * TN;
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                const int p = p0 + kGroup * j;
                v[g][j] = (cc <= c_hi && p < npairs) ? __ldcg(reinterpret_cast<const longlong2*>(base) + p)
                                                     : make_longlong2(0, 0);
              }
            }
#pragma unroll
            for (int g = 0; g < 4; ++g)
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                acc[j].x += v[g][j].x;
                acc[j].y += v[g][j].y;
              }
          }
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int p = p0 + kGroup * j;
            if (p >= npairs) break;
            const int mm = p / (TN / 2), col = 2 * (p % (TN / 2)), n = t * TN + col;
            const int em = s.row_exp[mm];
            if (n < a.N) store_i8(a, mm, n, acc[j].x, em, s.tscale[col]);
            if (n + 1 < a.N) store_i8(a, mm, n + 1, acc[j].y, em, s.tscale[col + 1]);
          }
        }
      }
    }
  }

  if constexpr (kCluster) {
    // CTA `rank` owns columns [rank R, rank R + R) of the tile; every CTA of the cluster has stored its
    // exact partial sums of them into this CTA's slots. Integer sums: the order does not matter.
    cluster_sync_unaligned();  // release / acquire: every remote store has landed
    const int S = a.S;
    const int R = (TN + S - 1) / S;
    const int r0 = rank * R;
    const int ncols = r0 >= TN ? 0 : (r0 + R <= TN ? R : TN - r0);
    const int t = static_cast<int>(cluster_id_x());
    if (!*abort) {
      for (int item = threadIdx.x; item < ncols * a.M; item += kThreads) {
        const int mm = item / ncols, lc = item - mm * ncols;
        long long v = 0;
        for (int src = 0; src < S; ++src) v += s.red[(src * kRows + mm) * R + lc];
        const int n = t * TN + r0 + lc;
        if (n < a.N) store_i8(a, mm, n, v, s.row_exp[mm], __bfloat162float(a.scale[n]));
      }
    }
  }

  tc_fence_before_sync();
  cta_teardown_barrier();  // every thread has finished with TMEM before warp 1 frees it
  if (warp == 1) {
    tc_fence_after_sync();
    tmem_dealloc(tmem, Cfg::kTmemCols);
  }
}

template <typename T>
int ensure_smem_attr(T kernel, size_t bytes, bool* done) {
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && done[dev]) return BP_OK;
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(bytes));
  if (e != cudaSuccess) return fail(BP_ERR_CUDA, "cudaFuncSetAttribute(smem %zu): %s", bytes, cudaGetErrorString(e));
  if (dev >= 0 && dev < 64) done[dev] = true;
  return BP_OK;
}

// Work partition; depends on (N, K) and the SM count only, never on M.
struct I8Partition {
  int tn;           // tile rows: 256 (stream-K) or 128 (cluster mode)
  int tiles, kblocks, P, S;
  long long units;
};

I8Partition i8_partition(int N, int K) {
  I8Partition p;
  const int sms = tc_sm_count();
  p.kblocks = (K + kBK - 1) / kBK;
  const int tiles128 = (N + 127) / 128;
  if (2 * tiles128 <= sms) {
    // few tiles: 128-row tiles, each tile's K range split over a cluster of S CTAs
    p.tn = 128;
    p.tiles = tiles128;
    int S = 2 * sms / p.tiles;  // two CTAs fit per SM: two producers per SM (as in the bf16 kernel)
    if (S > kMaxClusterSplit) S = kMaxClusterSplit;
    if (S > p.kblocks) S = p.kblocks;
    p.S = S < 1 ? 1 : S;
    p.P = p.tiles * p.S;
  } else {
    p.tn = 256;
    p.tiles = (N + 255) / 256;
    p.S = 0;
    p.P = 0;
  }
  p.units = static_cast<long long>(p.tiles) * p.kblocks;
  if (p.S == 0) p.P = static_cast<int>(p.units < sms ? p.units : sms);
  return p;
}

template <int TN, bool kCluster>
cudaError_t launch_main(cudaLaunchConfig_t* cfg, const CUtensorMap& tw, const CUtensorMap& ta, const I8Args& a) {
  static bool done[64] = {false};
  if (ensure_smem_attr(skinny_i8_kernel<TN, kCluster>, smem_bytes<TN>(), done) != BP_OK) return cudaErrorInvalidValue;
  cfg->dynamicSmemBytes = smem_bytes<TN>();
  return cudaLaunchKernelEx(cfg, skinny_i8_kernel<TN, kCluster>, tw, ta, a);
}

// Workspace: tile counters, row exponents, the digit matrix (up to 64 rows of K bytes), the partials.
size_t digit_bytes(int K) { return (static_cast<size_t>(kAM) * K + 1023) & ~static_cast<size_t>(1023); }

}  // namespace

size_t skinny_i8_workspace_bytes(int N, int K) {
  if (N <= 0 || K <= 0) return 0;
  const I8Partition p = i8_partition(N, K);
  const size_t head = kTcCountersBytes + kExpBytes + digit_bytes(K);
  if (p.S > 0) return head;
  return head + static_cast<size_t>(p.P) * 2 * kRows * p.tn * sizeof(long long);
}

bool skinny_i8_supported(const void* x, long long ldx, const void* w, int M, int N, int K) {
  const bool al = (reinterpret_cast<uintptr_t>(x) & 15u) == 0 && (reinterpret_cast<uintptr_t>(w) & 15u) == 0;
  return al && K >= 16 && K % 16 == 0 && K <= 131072 && M >= 1 && M <= kRows && N >= 1 &&
         (N + 127) / 128 <= kTcMaxTiles && ldx % 8 == 0;
}

int launch_skinny_i8(const void* x, long long ldx, const void* w, const void* w_scale, void* y, long long ldy, int y_f32,
                     int M, int N, int K, void* ws, size_t ws_bytes, cudaStream_t stream) {
  const I8Partition p = i8_partition(N, K);
  const size_t need = skinny_i8_workspace_bytes(N, K);
  if (ws == nullptr || ws_bytes < need)
    return fail(BP_ERR_INVALID_ARGUMENT, "the int8 tensor-core path needs a zero-initialised workspace of %zu bytes (got %zu)",
                need, ws_bytes);
  if ((reinterpret_cast<uintptr_t>(ws) & 255u) != 0) return fail(BP_ERR_MISALIGNED, "workspace must be 256-byte aligned");
  int* exps = reinterpret_cast<int*>(static_cast<char*>(ws) + kTcCountersBytes);
  uint8_t* digits = reinterpret_cast<uint8_t*>(static_cast<char*>(ws) + kTcCountersBytes + kExpBytes);
  CUtensorMap tw, ta;
  int st = tc_encode_2d(&tw, CU_TENSOR_MAP_DATA_TYPE_UINT8, w, static_cast<uint64_t>(K), static_cast<uint64_t>(N),
                        static_cast<uint64_t>(K), kBK, static_cast<uint32_t>(p.tn), CU_TENSOR_MAP_L2_PROMOTION_L2_256B);
  if (st != BP_OK) return st;
  // the digit matrix has 4 M rows: the tile's rows beyond them are zero-filled
  st = tc_encode_2d(&ta, CU_TENSOR_MAP_DATA_TYPE_UINT8, digits, static_cast<uint64_t>(K), static_cast<uint64_t>(4 * M),
                    static_cast<uint64_t>(K), kBK, kAM, CU_TENSOR_MAP_L2_PROMOTION_L2_128B);
  if (st != BP_OK) return st;

  cudaLaunchAttribute pdl[1];
  int npdl = 0;
  if (tc_pdl_enabled()) {
    pdl[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    pdl[0].val.programmaticStreamSerializationAllowed = 1;
    npdl = 1;
  }
  // 1. row exponents and digits
  {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(M, 1, 1);
    cfg.blockDim = dim3(256, 1, 1);
    cfg.stream = stream;
    cfg.attrs = pdl;
    cfg.numAttrs = npdl;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, i8_digitise_kernel, static_cast<const __nv_bfloat16*>(x), ldx, K,
                                             exps, digits);
    if (e != cudaSuccess) return fail(BP_ERR_CUDA, "int8 digitise launch (M=%d K=%d): %s", M, K, cudaGetErrorString(e));
  }
  // 2. the weight stream
  I8Args a;
  a.y = y;
  a.ldy = ldy;
  a.y_f32 = y_f32;
  a.scale = static_cast<const __nv_bfloat16*>(w_scale);
  a.exps = exps;
  a.M = M;
  a.N = N;
  a.K = K;
  a.tiles = p.tiles;
  a.kblocks = p.kblocks;
  a.units = p.units;
  a.P = p.P;
  a.S = p.S;
  a.counters = static_cast<int*>(ws);
  a.partials = reinterpret_cast<long long*>(static_cast<char*>(ws) + kTcCountersBytes + kExpBytes + digit_bytes(K));

  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.P, 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  int na = 0;
  if (npdl) attr[na++] = pdl[0];
  if (p.S > 0) {
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = p.S;
    attr[na].val.clusterDim.y = 1;
    attr[na].val.clusterDim.z = 1;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  const cudaError_t e = p.S > 0 ? launch_main<128, true>(&cfg, tw, ta, a) : launch_main<256, false>(&cfg, tw, ta, a);
  if (e != cudaSuccess)
    return fail(BP_ERR_CUDA, "int8 tensor-core skinny launch (M=%d N=%d K=%d P=%d S=%d): %s", M, N, K, p.P, p.S,
                cudaGetErrorString(e));
  return BP_OK;
}

BP_DEFINE_DEVICE_ERROR_READER(read_device_errors_i8)

}  // namespace bp
