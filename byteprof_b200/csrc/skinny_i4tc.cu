// Tensor-core skinny linear with int4 group-128 weights in byteprof's tile-major format, M <= 16
// activation rows per launch:
//   y[m, n] = sum_g scale[g, n] * (sum_{k in g} q[n, k] x[m, k] - zero[g, n] * sum_{k in g} x[m, k]).
//
// Reference: byteprof/optim/skinny.py:1-19 (the format), 46-63 (_skinny_kernel MODE 3: per group, q - zero
// times x summed in fp32 and the group scale applied to that partial) and 136-166 (skinny_mm).
//
// B200 design. The CUDA-core kernel (skinny_i4.cu) reads four bytes of staged activations from shared
// memory per weight and is bound by that at every M; here the tensor cores do the reuse.
//  * Swap-AB integer MMA (kind::i8): a 128-row weight tile with its codes unpacked to one byte each is the
//    A operand (M = 128); the activations written exactly as four signed base-256 digit planes
//    (digits.cuh) are B (N = 4 M rounded up to 16, rows beyond 4 M zero). Codes are 0..15, so A is a valid
//    s8 operand, and the int32 sums S_p = sum_k q d_p are exact (|S_p| <= 128 * 15 * 128 < 2^18).
//  * Per group: four MMAs (K = 32) into a fresh TMEM accumulator of 4 M int32 columns (a ring of four).
//    The epilogue thread of weight row n reads its row's plane sums, forms T = sum_p 2^(8 p) S_p
//    (= sum_k q X) in fp32 and adds scale (T - zero Xg) to its fp32 accumulator, with Xg = sum_k X of the
//    group from the prep kernel; 2^(e_m - 29) scales the tile's result once at the end.
//  * A unit is (128-row tile, GB consecutive groups), GB in {1, 2, 4} chosen from (N, K): issuing a copy
//    costs a few hundred cycles whatever its size, so each unit's data comes in five copies: one 4-D TMA
//    box of packed codes (GB groups x the four 2 KB blocks of the format's 32-row tiles, L2
//    evict-first), one 2-D box each of scale and zero rows, one 3-D box of digit tiles (the workspace
//    holds the digits group-major) and one bulk copy of the group sums. Blocks past the last row tile or
//    group are zero-filled by TMA.
//  * The weight and digit rings are fixed shared-memory regions cut into stages of GB groups at run time
//    (96 KB of packed codes: 3, 6 or 12 stages; 64 KB of digit tiles: 2 to 32 stages). A digit tile comes
//    from L2 but lands behind the weight boxes of the SM's copy queue, about 2 us after it is requested,
//    so the digit ring must run many groups ahead of the MMAs.
//  * Warp roles: 0 weight copies; 1 MMA issue and TMEM owner; 2-5 epilogue (warp w reads TMEM lanes
//    32 (w % 4) ..); 6-9 unpack, each warp a whole group in turn (group j to warp j % W, W = 4, or 3 with
//    three unpacked-tile slots), the nibbles into
//    the 128-byte-swizzled K-major layout the MMA reads (bytes 0-63 of a row are the low nibbles and
//    64-127 the high ones, as in the format); 10 digit copies, once the prep kernel has finished.
//  * Every barrier operation and tcgen05 instruction costs the issuing thread some 50-150 cycles, so the
//    MMA warp and the epilogue synchronise per unit: a unit's GB accumulators sit side by side in one of
//    two TMEM buffers, with one commit and one release per unit.
//  * Stream-K over the tiles x groups/GB units on one CTA per SM, from (N, K) only: a tile split between
//    CTAs is finished by the CTA that arrives last, adding the partials in CTA order (deterministic; a
//    row's result depends neither on M nor on the other rows).
//  * A prep kernel writes the row exponents, the digit matrix and the group sums Xg into the workspace;
//    programmatic dependent launch lets the main kernel's weight copies start under it.
//  * Every mbarrier wait is bounded (2 s, then the device error word, a drain of the copies in flight,
//    TMEM freed, return).
#include <cudaTypedefs.h>
#include <cuda_fp16.h>

#include "digits.cuh"
#include "skinny_internal.h"
#include "sm100.cuh"

namespace bp {
namespace {

constexpr int kGroup = 128;                     // K per group = one 128-byte row of unpacked codes
constexpr int kBM = 128;                        // weight rows per tile (MMA M)
constexpr int kFmtRows = 32;                    // rows per tile of the packed format
constexpr int kFmtBlock = kFmtRows * 64;        // 2 KB: one format tile x one group
constexpr int kGroupPacked = kBM * 64;          // 8 KB of packed codes per tile and group
constexpr int kUnpackedBytes = kBM * kGroup;    // 16 KB per tile and group
constexpr int kGBMax = 4;                       // groups per unit
constexpr int kRows = 16;                       // activation rows per launch
constexpr int kPackedRegion = 3 * kGBMax * kGroupPacked;  // 96 KB: GB-group weight stages
constexpr int kWSlots = kPackedRegion / kGroupPacked;     // 12 group slots of scale and zero rows
template <int kNB>
constexpr int a_slots() {  // unpacked tiles (groups)
  return kNB <= 32 ? 5 : 3;
}
// Unpack warps in use: at most the number of unpacked-tile slots. A warp waits for its slot to be free
// only once per group it takes, so the wait for group j is known to follow the release of group
// j - warps - slots; with warps <= slots that is at least group j - 2 slots, and the slot's parity wait
// cannot be satisfied by a release two uses old.
template <int kNB>
constexpr int unpack_warps() {
  return a_slots<kNB>() < 4 ? a_slots<kNB>() : 4;
}
template <int kNB>
constexpr int digit_slots() {  // groups of digit tiles: 32 KB (64 KB for 48 and 64 digit rows)
  return (kNB <= 32 ? 32 * 1024 : 64 * 1024) / (kNB * kGroup);
}
constexpr int kThreads = 352;                   // 11 warps
constexpr int kEpiWarp0 = 2;
constexpr int kUnpackWarp0 = 6;
constexpr int kDigitWarp = 10;
constexpr int kEpiThreads = 128;
constexpr size_t kExpBytes = 1024;

struct I4Args {
  void* y;
  long long ldy;
  int y_f32;
  const int* exps;               // [kRows] row exponents (workspace)
  const float* xg;               // [G][kRows] group sums of the fixed-point activations (workspace)
  int M, N, G, GB, UG;           // UG = ceil(G / GB) units per tile
  int WSU, DSU;                  // weight and digit stages of GB groups
  long long units;
  int P;
  int* counters;                 // [tiles], zero between launches
  float* partials;               // [P][2][kRows][kBM]
};

template <int kNB>
struct __align__(1024) I4Smem {
  static constexpr int kDSlots = digit_slots<kNB>();
  static constexpr int kAS = a_slots<kNB>();
  uint8_t ua[kAS][kUnpackedBytes];               // unpacked codes, the MMA's A operand (1024-byte aligned)
  uint8_t bd[kDSlots][kNB * kGroup];             // digit tiles, the B operand (1024-byte aligned)
  uint8_t packed[kPackedRegion];                 // stage st: [row tile][group][2 KB] as the 4-D box lands
  uint16_t sc[kWSlots][kBM];                     // scale (bf16 bits) [group slot][row]
  uint16_t zr[kWSlots][kBM];                     // zero (fp16 bits) [group slot][row]
  alignas(16) float xs[kDSlots][kRows];
  uint64_t full[kWSlots], empty[kWSlots];
  uint64_t afull[kAS], aempty[kAS];
  uint64_t dfull[kDSlots], dempty[kDSlots];
  uint64_t tfull[2], tempty[2];
  uint64_t mma_done;
  int row_exp[kRows];
  uint32_t tmem_base;
  int abort;
  int last_flag;
};
template <int kNB>
constexpr size_t smem_bytes() {
  return sizeof(I4Smem<kNB>) + 1024;  // + slack to align the base to 1024 bytes
}
static_assert(smem_bytes<64>() <= 232448, "shared memory per CTA");
template <int kNB>
constexpr uint32_t tmem_stride() {  // columns per group accumulator
  return kNB <= 16 ? 16u : (kNB <= 32 ? 32u : 64u);
}
template <int kNB>
constexpr uint32_t tmem_unit() {  // columns per unit buffer (kGBMax accumulators)
  return kGBMax * tmem_stride<kNB>();
}
template <int kNB>
constexpr uint32_t tmem_cols() {  // two unit buffers: 128, 256 or 512 columns
  return 2 * tmem_unit<kNB>();
}

__host__ __device__ __forceinline__ long long unit_start(int c, long long U, int P) {
  return static_cast<long long>(c) * U / P;
}
__host__ __device__ __forceinline__ int unit_owner(long long u, long long U, int P) {
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

// 1-D bulk copy global -> this CTA's shared memory, completing `bytes` on the mbarrier.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
               ::"r"(smem_addr(dst)), "l"(src), "r"(bytes), "r"(smem_addr(bar))
               : "memory");
}

// 32 lanes x 16 TMEM columns into r[0..15], without waiting.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, "
      "[%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
// Ties 16 registers to a point in the instruction stream (after tcgen05.wait::ld), so that no use of
// them is scheduled before the wait.
__device__ __forceinline__ void reg_fence16(uint32_t* r) {
  asm volatile(""
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                 "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                 "+r"(r[15]));
}
template <int kNB>
__device__ __forceinline__ void tmem_ld_cols(uint32_t taddr, uint32_t (&r)[kNB]) {
#pragma unroll
  for (int c = 0; c < kNB / 16; ++c) tmem_ld16(taddr + 16 * c, &r[16 * c]);
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int c = 0; c < kNB / 16; ++c) reg_fence16(&r[16 * c]);
}

// An int32 of magnitude below 2^22 as fp32 (exact): its bits added into the mantissa of 1.5 * 2^23.
__device__ __forceinline__ float small_int_to_float(uint32_t v) {
  return __uint_as_float(v + 0x4B400000u) - 12582912.0f;
}

__device__ __forceinline__ void store_value(const I4Args& a, int m, int row, float v) {
  if (a.y_f32)
    static_cast<float*>(a.y)[m * a.ldy + row] = v;
  else
    static_cast<__nv_bfloat16*>(a.y)[m * a.ldy + row] = __float2bfloat16_rn(v);
}

// Row exponents, the digit matrix [G][4 M][128] (group-major: one group's planes of all rows are one
// contiguous tile) and the group sums Xg[g][m] = sum_{k in g} X[m, k] (exact in int64, rounded once to
// fp32) of the M activation rows, one CTA per row. Values k = base + 1024 j + 8 t (t the thread) are one
// 16-byte chunk; each half-warp covers one group. The first 4096 values stay in registers between the
// exponent pass and the digit pass.
// The CTA is small (128 threads, at most 40 registers each) so that it fits on an SM beside a CTA of the
// main kernel (352 threads x 168 registers of the SM's 65536): launched early, it must not hold an SM
// that the main kernel's CTAs need, or the CTA left without one starts only when this kernel has ended.
constexpr int kPrepThreads = 128;
__global__ void __launch_bounds__(kPrepThreads, 12) i4_prep_kernel(const __nv_bfloat16* x, long long ldx, int M, int K,
                                                                int* exps, uint8_t* digits, float* xg) {
  constexpr int kChunk = 8 * kPrepThreads;  // values per chunk row of the CTA
  constexpr int kPass = 4 * kChunk;
  pdl_launch_dependents();  // the main kernel may start streaming weights now
  pdl_wait_prior_grids();   // x may come from the previous kernel
  const int m = blockIdx.x;
  const int lane = threadIdx.x & 31;
  const __nv_bfloat16* xr = x + static_cast<long long>(m) * ldx;
  uint32_t amax = 0;
  uint4 keep[4];
  for (int base = 0; base < K; base += kPass) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int k = base + kChunk * j + 8 * static_cast<int>(threadIdx.x);
      const uint4 v = k < K ? __ldcg(reinterpret_cast<const uint4*>(xr + k)) : make_uint4(0, 0, 0, 0);
      if (base == 0) keep[j] = v;
      const uint32_t wv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int h = 0; h < 4; ++h) amax = max(amax, max(wv[h] & 0x7fffu, (wv[h] >> 16) & 0x7fffu));
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = max(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  __shared__ uint32_t red[kPrepThreads / 32];
  __shared__ int e_row;
  if (lane == 0) red[threadIdx.x >> 5] = amax;
  __syncthreads();
  if (threadIdx.x == 0) {
    uint32_t mx = 0;
    for (int w = 0; w < kPrepThreads / 32; ++w) mx = max(mx, red[w]);
    e_row = row_exponent(mx);
    exps[m] = e_row;
  }
  __syncthreads();
  const bool nonfinite = e_row == kNonFinite;  // the row's output is NaN; its digits and sums are zero
  const int e = nonfinite ? 0 : e_row;
  for (int base = 0; base < K; base += kPass) {  // the loop bound is uniform over the CTA
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int k = base + kChunk * j + 8 * static_cast<int>(threadIdx.x);
      const bool in = k < K;  // uniform over each half-warp (K is a multiple of 128)
      uint4 v = base == 0 ? keep[j] : (in ? __ldcg(reinterpret_cast<const uint4*>(xr + k)) : make_uint4(0, 0, 0, 0));
      if (nonfinite) v = make_uint4(0, 0, 0, 0);
      uint32_t pl[kDigitPlanes][2];
      long long sum = digitise8(v, e, pl);
      const int g = k / kGroup, kk = k % kGroup;
      if (in) {
#pragma unroll
        for (int p = 0; p < kDigitPlanes; ++p)
          *reinterpret_cast<uint2*>(digits + (static_cast<size_t>(g) * 4 * M + 4 * m + p) * kGroup + kk) =
              make_uint2(pl[p][0], pl[p][1]);
      }
#pragma unroll
      for (int o = 1; o < 16; o <<= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
      if (in && (lane & 15) == 0) xg[g * kRows + m] = __ll2float_rn(sum);
    }
  }
}

template <int kNB>
__global__ void __launch_bounds__(kThreads, 1)
    skinny_i4tc_kernel(const __grid_constant__ CUtensorMap tw, const __grid_constant__ CUtensorMap tsc,
                       const __grid_constant__ CUtensorMap tzr, const __grid_constant__ CUtensorMap td,
                       const I4Args a) {
  constexpr int kMR = kNB / 4;  // activation rows this instantiation computes (>= M)
  constexpr int kAS = a_slots<kNB>();
  extern __shared__ uint8_t smem_raw[];
  I4Smem<kNB>& s =
      *reinterpret_cast<I4Smem<kNB>*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int c = blockIdx.x;
  const long long U = a.units;
  const int G = a.G, GB = a.GB, UG = a.UG, WSU = a.WSU, DSU = a.DSU;
  const long long u0 = unit_start(c, U, a.P);
  const long long u1 = unit_start(c + 1, U, a.P);
  const int n_units = static_cast<int>(u1 - u0);

  if (threadIdx.x == 0) {
    for (int i = 0; i < WSU; ++i) {
      mbar_init(&s.full[i], 1);
      mbar_init(&s.empty[i], GB + 4);  // GB from the unpack warps and one from each epilogue warp
    }
    for (int i = 0; i < kAS; ++i) {
      mbar_init(&s.afull[i], 32);  // the lanes of the unpacking warp
      mbar_init(&s.aempty[i], 1);
    }
    for (int i = 0; i < DSU; ++i) {
      mbar_init(&s.dfull[i], 1);
      mbar_init(&s.dempty[i], 1 + 4);  // the MMA commit and the four epilogue warps
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&s.tfull[b], 1);
      mbar_init(&s.tempty[b], kEpiThreads);
    }
    mbar_init(&s.mma_done, 1);
    s.abort = 0;
    s.last_flag = 0;
    mbar_fence_init();
    tma_prefetch_desc(&tw);
    tma_prefetch_desc(&tsc);
    tma_prefetch_desc(&tzr);
    tma_prefetch_desc(&td);
  }
  if (warp == 1) {
    tmem_alloc(&s.tmem_base, tmem_cols<kNB>());
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
      // ---- packed codes, scale and zero rows of a unit: three TMA boxes, independent of earlier kernels ----
      const uint64_t pol = l2_evict_first_policy();
      const uint32_t bytes = static_cast<uint32_t>(GB * (kGroupPacked + 2 * kBM * 2));
      int issued = 0;
      for (int i = 0; i < n_units; ++i) {
        const int st = i % WSU;
        if (i >= WSU && !mbar_wait(&s.empty[st], static_cast<uint32_t>((i / WSU) + 1) & 1u, abort)) break;
        const long long u = u0 + i;
        const int t = static_cast<int>(u / UG), g0 = static_cast<int>(u % UG) * GB;
        mbar_arrive_expect_tx(&s.full[st], bytes);
        tma_load_4d_hint(s.packed + st * GB * kGroupPacked, &tw, &s.full[st], 0, 0, g0, 4 * t, pol);
        tma_load_2d_hint(s.sc[st * GB], &tsc, &s.full[st], t * kBM, g0, pol);
        tma_load_2d_hint(s.zr[st * GB], &tzr, &s.full[st], t * kBM, g0, pol);
        issued = i + 1;
      }
      for (int st = 0; st < WSU && st < issued; ++st) {  // drain
        const int i_last = st + WSU * ((issued - 1 - st) / WSU);
        wait_drain(&s.full[st], static_cast<uint32_t>(i_last / WSU) & 1u);
      }
    }
  } else if (warp == kDigitWarp) {
    if (lane == 0) {
      // ---- digit tiles and group sums of a unit: written by the prep kernel ----
      pdl_wait_prior_grids();
      int issued = 0;
      for (int i = 0; i < n_units; ++i) {
        const int ds = i % DSU;
        if (i >= DSU && !mbar_wait(&s.dempty[ds], static_cast<uint32_t>((i / DSU) + 1) & 1u, abort)) break;
        const int g0 = static_cast<int>((u0 + i) % UG) * GB;
        const int ng = G - g0 < GB ? G - g0 : GB;
        mbar_arrive_expect_tx(&s.dfull[ds], static_cast<uint32_t>(GB * kNB * kGroup + ng * kRows * 4));
        tma_load_3d(s.bd[ds * GB], &td, &s.dfull[ds], 0, 0, g0);
        bulk_g2s(s.xs[ds * GB], a.xg + static_cast<long long>(g0) * kRows, static_cast<uint32_t>(ng * kRows * 4),
                 &s.dfull[ds]);
        issued = i + 1;
      }
      for (int ds = 0; ds < DSU && ds < issued; ++ds) {  // drain
        const int i_last = ds + DSU * ((issued - 1 - ds) / DSU);
        wait_drain(&s.dfull[ds], static_cast<uint32_t>(i_last / DSU) & 1u);
      }
    }
  } else if (warp >= kUnpackWarp0) {
    // ---- unpack: packed row r (64 bytes) -> unpacked row r (128 bytes, 128-byte swizzle) ----
    // Warp uw unpacks groups j = uw, uw + kUW, ... Lane l handles 16-byte chunk cp of the packed rows
    // r = 32 it + 8 a + rsel (it, a = 0..3): the eight lanes of each shared-memory phase take rows r and
    // r ^ 5 (four chunks each), so their reads fall in both halves of the banks and their swizzled stores
    // in both halves of the row.
    constexpr int kUW = unpack_warps<kNB>();
    const int uw = warp - kUnpackWarp0;
    const int i8 = lane & 7, pi = (lane >> 3) & 3;
    const int rsel = i8 < 4 ? pi : (pi ^ 5);
    const int cp = i8 & 3;
    const int src_off = rsel * 64 + cp * 16;
    const int lo_off = rsel * kGroup + ((cp ^ rsel) << 4);
    const int hi_off = rsel * kGroup + (((cp + 4) ^ rsel) << 4);
    int j = 0;  // group sequence number
    bool ok = true;
    for (int i = 0; i < n_units && ok && uw < kUW; ++i) {
      const int st = i % WSU;
      const int g0 = static_cast<int>((u0 + i) % UG) * GB;
      const int ng = G - g0 < GB ? G - g0 : GB;
      bool have_stage = false;
      for (int gg = 0; gg < ng; ++gg, ++j) {
        if (j % kUW != uw) continue;
        if (!have_stage) {
          if (!mbar_wait(&s.full[st], static_cast<uint32_t>(i / WSU) & 1u, abort)) {
            ok = false;
            break;
          }
          have_stage = true;
        }
        const int as = j % kAS;
        if (j >= kAS && !mbar_wait(&s.aempty[as], static_cast<uint32_t>((j / kAS) + 1) & 1u, abort)) {
          ok = false;
          break;
        }
        const uint8_t* src = s.packed + st * GB * kGroupPacked + gg * kFmtBlock + src_off;
        uint8_t* dst = s.ua[as];
#pragma unroll
        for (int it = 0; it < kBM / kFmtRows; ++it) {
#pragma unroll
          for (int aa = 0; aa < 4; ++aa) {
            const uint4 v = *reinterpret_cast<const uint4*>(src + it * GB * kFmtBlock + aa * 8 * 64);
            const uint4 lo = make_uint4(v.x & 0x0F0F0F0Fu, v.y & 0x0F0F0F0Fu, v.z & 0x0F0F0F0Fu, v.w & 0x0F0F0F0Fu);
            const uint4 hi = make_uint4((v.x >> 4) & 0x0F0F0F0Fu, (v.y >> 4) & 0x0F0F0F0Fu, (v.z >> 4) & 0x0F0F0F0Fu,
                                        (v.w >> 4) & 0x0F0F0F0Fu);
            const int ro = (it * kFmtRows + aa * 8) * kGroup;
            *reinterpret_cast<uint4*>(dst + ro + lo_off) = lo;
            *reinterpret_cast<uint4*>(dst + ro + hi_off) = hi;
          }
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // visible to the MMA's operand reads
        mbar_arrive(&s.afull[as]);
        __syncwarp();
        // the stage is released after all GB groups: the last group's warp arrives for the missing ones
        if (lane == 0)
          for (int k = (gg == ng - 1 ? GB - ng + 1 : 1); k > 0; --k) mbar_arrive(&s.empty[st]);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---- MMA issuer: per group 4 x (M 128, N kNB, K 32) into a fresh accumulator; per unit one buffer ----
      constexpr uint32_t idesc = umma_idesc_s8(kBM, kNB);
      int j = 0;
      bool ok = true;
      for (int i = 0; i < n_units && ok; ++i) {
        const int ds = i % DSU, ub = i & 1;
        const int g0 = static_cast<int>((u0 + i) % UG) * GB;
        const int ng = G - g0 < GB ? G - g0 : GB;
        if (!mbar_wait(&s.dfull[ds], static_cast<uint32_t>(i / DSU) & 1u, abort)) break;
        if (i >= 2 && !mbar_wait(&s.tempty[ub], static_cast<uint32_t>((i >> 1) + 1) & 1u, abort)) break;
        const uint32_t dbase = tmem + static_cast<uint32_t>(ub) * tmem_unit<kNB>();
        for (int gg = 0; gg < ng; ++gg, ++j) {
          const int as = j % kAS;
          if (!mbar_wait(&s.afull[as], static_cast<uint32_t>(j / kAS) & 1u, abort)) {
            ok = false;
            break;
          }
          tc_fence_after_sync();
          const uint64_t ad = umma_desc_sw128(smem_addr(s.ua[as]));
          const uint64_t bd = umma_desc_sw128(smem_addr(s.bd[ds * GB + gg]));
          const uint32_t d = dbase + static_cast<uint32_t>(gg) * tmem_stride<kNB>();
#pragma unroll
          for (int kk = 0; kk < kGroup / 32; ++kk)  // +32 bytes along K = +2 in the descriptor's address field
            umma_i8(d, ad + 2 * kk, bd + 2 * kk, idesc, kk > 0 ? 1u : 0u);
          umma_commit(&s.aempty[as]);  // the unpacked tile is free once these MMAs have read it
        }
        if (!ok) break;
        umma_commit(&s.tfull[ub]);
        umma_commit(&s.dempty[ds]);  // the unit's digit tiles are read
      }
      umma_commit(&s.mma_done);
      wait_drain(&s.mma_done, 0);
    }
  } else {
    // ---- epilogue: per group, TMEM -> fp32 accumulators; per tile, y (or a stream-K partial) ----
    pdl_wait_prior_grids();
    const int q = warp & 3;  // TMEM lane quadrant this warp may access
    const int r = 32 * q + lane;
    const int et = threadIdx.x - 32 * kEpiWarp0;
    if (et < kRows) s.row_exp[et] = et < a.M ? __ldcg(a.exps + et) : 0;
    named_barrier_sync(1, kEpiThreads);
    int ex[kMR];
    float acc[kMR];
#pragma unroll
    for (int m = 0; m < kMR; ++m) {
      ex[m] = s.row_exp[m];
      acc[m] = 0.0f;
    }
    const int t_first = static_cast<int>(u0 / UG);
    bool ok = true;
    for (int i = 0; i < n_units; ++i) {
      const long long u = u0 + i;
      const int t = static_cast<int>(u / UG), g0 = static_cast<int>(u % UG) * GB;
      const int ng = G - g0 < GB ? G - g0 : GB;
      const int st = i % WSU, ds = i % DSU;
      // this row's scale and zero of the unit's groups; the weight stage is then free of the epilogue
      ok = ok && mbar_wait(&s.full[st], static_cast<uint32_t>(i / WSU) & 1u, abort);
      float scv[kGBMax], nzv[kGBMax];
#pragma unroll
      for (int gg = 0; gg < kGBMax; ++gg) {
        scv[gg] = (ok && gg < ng) ? __uint_as_float(static_cast<uint32_t>(s.sc[st * GB + gg][r]) << 16) : 0.0f;
        nzv[gg] = (ok && gg < ng) ? -__half2float(__ushort_as_half(s.zr[st * GB + gg][r])) : 0.0f;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&s.empty[st]);
      ok = ok && mbar_wait(&s.dfull[ds], static_cast<uint32_t>(i / DSU) & 1u, abort);
      const float* xsu = s.xs[ds * GB];
      const int ub = i & 1;
      ok = ok && mbar_wait(&s.tfull[ub], static_cast<uint32_t>(i >> 1) & 1u, abort);
      ok = __all_sync(0xffffffffu, ok);  // the TMEM loads below are warp-collective
      if (ok) tc_fence_after_sync();
      const uint32_t tbase = tmem + (static_cast<uint32_t>(32 * q) << 16) + static_cast<uint32_t>(ub) * tmem_unit<kNB>();
#pragma unroll
      for (int gg = 0; gg < kGBMax; ++gg) {
        if (gg >= ng) break;
        uint32_t S[kNB];
        if (ok) {
          tmem_ld_cols<kNB>(tbase + static_cast<uint32_t>(gg) * tmem_stride<kNB>(), S);
        } else {
#pragma unroll
          for (int jj = 0; jj < kNB; ++jj) S[jj] = 0;
        }
#pragma unroll
        for (int m = 0; m < kMR; ++m) {
          float T = fmaf(small_int_to_float(S[4 * m + 1]), 256.0f, small_int_to_float(S[4 * m]));
          T = fmaf(small_int_to_float(S[4 * m + 2]), 65536.0f, T);
          T = fmaf(small_int_to_float(S[4 * m + 3]), 16777216.0f, T);
          acc[m] = fmaf(scv[gg], fmaf(nzv[gg], xsu[gg * kRows + m], T), acc[m]);
        }
      }
      tc_fence_before_sync();
      mbar_arrive(&s.tempty[ub]);
      __syncwarp();
      if (lane == 0) mbar_arrive(&s.dempty[ds]);
      if (g0 + ng != G && u != u1 - 1) continue;

      // ---- the tile's last group in this CTA ----
      if (named_barrier_or(1, kEpiThreads, !ok)) break;  // every epilogue thread takes the same decision
      float v[kMR];
#pragma unroll
      for (int m = 0; m < kMR; ++m) {
        v[m] = ex[m] == kNonFinite ? __int_as_float(0x7fffffff) : ldexpf(acc[m], ex[m] - kFracBits);
        acc[m] = 0.0f;
      }
      const int row = t * kBM + r;
      const int c_lo = unit_owner(static_cast<long long>(t) * UG, U, a.P);
      const int c_hi = unit_owner(static_cast<long long>(t + 1) * UG - 1, U, a.P);
      if (c_lo == c_hi) {
        if (row < a.N)
#pragma unroll
          for (int m = 0; m < kMR; ++m)
            if (m < a.M) store_value(a, m, row, v[m]);
        continue;
      }
      const int slot = (t == t_first) ? 0 : 1;
      float* mine = a.partials + static_cast<size_t>(c * 2 + slot) * kRows * kBM;
#pragma unroll
      for (int m = 0; m < kMR; ++m)
        if (m < a.M) mine[m * kBM + r] = v[m];
      __syncwarp();
      named_barrier_sync(1, kEpiThreads);  // every partial of this CTA is written ...
      if (et == 0) {
        __threadfence();  // ... and (cumulatively) visible GPU-wide before the arrival is counted
        const int old = atomicAdd(&a.counters[t], 1);
        const int last = old == c_hi - c_lo;
        if (last) {
          a.counters[t] = 0;  // every contributor has arrived: ready for the next launch
          __threadfence();    // acquire side: the other contributors' partials are visible from here on
        }
        s.last_flag = last;
      }
      __syncwarp();
      named_barrier_sync(1, kEpiThreads);
      if (s.last_flag && row < a.N) {
        float sum[kMR];
#pragma unroll
        for (int m = 0; m < kMR; ++m) sum[m] = 0.0f;
        for (int cc = c_lo; cc <= c_hi; ++cc) {  // fixed order: the sum does not depend on arrival order
          const int cslot = (t == static_cast<int>(unit_start(cc, U, a.P) / UG)) ? 0 : 1;
          const float* p = a.partials + static_cast<size_t>(cc * 2 + cslot) * kRows * kBM;
#pragma unroll
          for (int m = 0; m < kMR; ++m)
            if (m < a.M) sum[m] += __ldcg(p + m * kBM + r);
        }
#pragma unroll
        for (int m = 0; m < kMR; ++m)
          if (m < a.M) store_value(a, m, row, sum[m]);
      }
    }
  }

  tc_fence_before_sync();
  cta_teardown_barrier();  // every thread has finished with TMEM before warp 1 frees it
  if (warp == 1) {
    tc_fence_after_sync();
    tmem_dealloc(tmem, tmem_cols<kNB>());
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

struct I4Maps {
  CUtensorMap w, sc, zr, d;
};

template <int kNB>
cudaError_t launch_main(cudaLaunchConfig_t* cfg, const I4Maps& mp, const I4Args& a) {
  static bool done[64] = {false};
  if (ensure_smem_attr(skinny_i4tc_kernel<kNB>, smem_bytes<kNB>(), done) != BP_OK) return cudaErrorInvalidValue;
  cfg->dynamicSmemBytes = smem_bytes<kNB>();
  return cudaLaunchKernelEx(cfg, skinny_i4tc_kernel<kNB>, mp.w, mp.sc, mp.zr, mp.d, a);
}

// Work partition; depends on (N, K) and the SM count only, never on M. Units of GB groups, the largest
// GB that still gives every SM two units or more.
struct I4Partition {
  int tiles, G, GB, UG, P;
  long long units;
};
I4Partition i4_partition(int N, int K) {
  I4Partition p;
  const int sms = tc_sm_count();
  p.tiles = (N + kBM - 1) / kBM;
  p.G = K / kGroup;
  for (p.GB = kGBMax;; p.GB /= 2) {
    p.UG = (p.G + p.GB - 1) / p.GB;
    p.units = static_cast<long long>(p.tiles) * p.UG;
    if (p.GB == 1 || p.units >= 2LL * sms) break;
  }
  p.P = static_cast<int>(p.units < sms ? p.units : sms);
  return p;
}

// Workspace: tile counters, row exponents, group sums [G][16], the digit matrix [G][4 M][128] (at most
// 64 K bytes), the partials [P][2][16][128].
size_t xg_bytes(int K) { return (static_cast<size_t>(K / kGroup) * kRows * 4 + 1023) & ~static_cast<size_t>(1023); }
size_t digit_bytes(int K) { return (static_cast<size_t>(kRows * kDigitPlanes) * K + 1023) & ~static_cast<size_t>(1023); }

}  // namespace

size_t skinny_i4tc_workspace_bytes(int N, int K) {
  if (N <= 0 || K <= 0 || K % kGroup != 0) return 0;
  const I4Partition p = i4_partition(N, K);
  return kTcCountersBytes + kExpBytes + xg_bytes(K) + digit_bytes(K) +
         static_cast<size_t>(p.P) * 2 * kRows * kBM * sizeof(float);
}

bool skinny_i4tc_supported(const void* x, long long ldx, const void* w, const void* scale, const void* zero, int M,
                           int N, int K) {
  const auto al = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  return al(x) && al(w) && al(scale) && al(zero) && ldx % 8 == 0 && N >= 8 && N % 8 == 0 && K >= kGroup &&
         K % kGroup == 0 && K <= 131072 && M >= 1 && M <= kRows && (N + kBM - 1) / kBM <= kTcMaxTiles;
}

int launch_skinny_i4tc(const void* x, long long ldx, const uint8_t* w, const void* scale, const void* zero, void* y,
                       long long ldy, int y_f32, int M, int N, int K, void* ws, size_t ws_bytes, cudaStream_t stream) {
  const I4Partition p = i4_partition(N, K);
  const size_t need = skinny_i4tc_workspace_bytes(N, K);
  if (ws == nullptr || ws_bytes < need)
    return fail(BP_ERR_INVALID_ARGUMENT, "the int4 tensor-core path needs a zero-initialised workspace of %zu bytes (got %zu)",
                need, ws_bytes);
  if ((reinterpret_cast<uintptr_t>(ws) & 255u) != 0) return fail(BP_ERR_MISALIGNED, "workspace must be 256-byte aligned");
  char* base = static_cast<char*>(ws);
  int* exps = reinterpret_cast<int*>(base + kTcCountersBytes);
  float* xg = reinterpret_cast<float*>(base + kTcCountersBytes + kExpBytes);
  uint8_t* digits = reinterpret_cast<uint8_t*>(base + kTcCountersBytes + kExpBytes + xg_bytes(K));
  float* partials = reinterpret_cast<float*>(base + kTcCountersBytes + kExpBytes + xg_bytes(K) + digit_bytes(K));
  const int nb = M <= 4 ? 16 : (M <= 8 ? 32 : (M <= 12 ? 48 : 64));
  const int RT = (N + kFmtRows - 1) / kFmtRows;

  I4Maps mp;
  {  // packed codes [RT][G][16][128 bytes]: x = byte in a 128-byte row, y = row pair, z = group, w = row tile
    const uint64_t dims[4] = {128, 16, static_cast<uint64_t>(p.G), static_cast<uint64_t>(RT)};
    const uint64_t strides[3] = {128, kFmtBlock, static_cast<uint64_t>(p.G) * kFmtBlock};
    const uint32_t box[4] = {128, 16, static_cast<uint32_t>(p.GB), 4};
    int st = tc_encode(&mp.w, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, w, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_NONE,
                       CU_TENSOR_MAP_L2_PROMOTION_L2_256B);
    if (st != BP_OK) return st;
  }
  {  // scale and zero [G][N] (16-bit): x = row n, y = group
    const uint64_t dims[2] = {static_cast<uint64_t>(N), static_cast<uint64_t>(p.G)};
    const uint64_t strides[1] = {static_cast<uint64_t>(N) * 2};
    const uint32_t box[2] = {kBM, static_cast<uint32_t>(p.GB)};
    int st = tc_encode(&mp.sc, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, scale, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_NONE,
                       CU_TENSOR_MAP_L2_PROMOTION_L2_256B);
    if (st != BP_OK) return st;
    st = tc_encode(&mp.zr, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, zero, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_NONE,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B);
    if (st != BP_OK) return st;
  }
  {  // digits [G][4 M][128]: a group's tile is nb rows (those beyond 4 M zero-filled) x 128 bytes
    const uint64_t dims[3] = {128, static_cast<uint64_t>(4 * M), static_cast<uint64_t>(p.G)};
    const uint64_t strides[2] = {128, static_cast<uint64_t>(4 * M) * 128};
    const uint32_t box[3] = {128, static_cast<uint32_t>(nb), static_cast<uint32_t>(p.GB)};
    int st = tc_encode(&mp.d, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, digits, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B,
                       CU_TENSOR_MAP_L2_PROMOTION_L2_128B);
    if (st != BP_OK) return st;
  }

  cudaLaunchAttribute pdl[1];
  int npdl = 0;
  if (tc_pdl_enabled()) {
    pdl[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    pdl[0].val.programmaticStreamSerializationAllowed = 1;
    npdl = 1;
  }
  {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(M, 1, 1);
    cfg.blockDim = dim3(kPrepThreads, 1, 1);
    cfg.stream = stream;
    cfg.attrs = pdl;
    cfg.numAttrs = npdl;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, i4_prep_kernel, static_cast<const __nv_bfloat16*>(x), ldx, M, K, exps,
                                             digits, xg);
    if (e != cudaSuccess) return fail(BP_ERR_CUDA, "int4 prep launch (M=%d K=%d): %s", M, K, cudaGetErrorString(e));
  }
  I4Args a;
  a.y = y;
  a.ldy = ldy;
  a.y_f32 = y_f32;
  a.exps = exps;
  a.xg = xg;
  a.M = M;
  a.N = N;
  a.G = p.G;
  a.GB = p.GB;
  a.UG = p.UG;
  a.WSU = kPackedRegion / (p.GB * kGroupPacked);
  const int dslots = nb == 16 ? digit_slots<16>() : nb == 32 ? digit_slots<32>() : nb == 48 ? digit_slots<48>() : digit_slots<64>();
  a.DSU = dslots / p.GB;
  a.units = p.units;
  a.P = p.P;
  a.counters = static_cast<int*>(ws);
  a.partials = partials;

  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.P, 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.stream = stream;
  cfg.attrs = pdl;
  cfg.numAttrs = npdl;
  cudaError_t e;
  switch (nb) {
    case 16: e = launch_main<16>(&cfg, mp, a); break;
    case 32: e = launch_main<32>(&cfg, mp, a); break;
    case 48: e = launch_main<48>(&cfg, mp, a); break;
    default: e = launch_main<64>(&cfg, mp, a); break;
  }
  if (e != cudaSuccess)
    return fail(BP_ERR_CUDA, "int4 tensor-core skinny launch (M=%d N=%d K=%d P=%d GB=%d): %s", M, N, K, p.P, p.GB,
                cudaGetErrorString(e));
  return BP_OK;
}

BP_DEFINE_DEVICE_ERROR_READER(read_device_errors_i4tc)

}  // namespace bp
