// Tensor-core skinny linear: y[M, N] = x[M, K] . W[N, K]^T for M <= 16 rows per launch, with bf16 weights
// or int8 weights and a per-row bf16 scale (y = scale[n] * sum_k q[n, k] x[m, k]).
//
// Reference: byteprof/optim/skinny.py:35-80 (_skinny_kernel MODE 0 / 1: one program per BN weight rows,
// swap-AB tl.dot with the weight tile as the MMA's M operand and the few activation rows as N; int8 widened
// to bf16 before tl.dot, scale applied to the accumulator) and skinny.py:83-90, 111-129 (split-K through
// an fp32 workspace and a second reduce kernel).
//
// B200 design:
//  * Swap-AB on the 5th-generation tensor cores: a 128-row weight tile is the A operand (MMA M = 128),
//    the activation rows padded to 16 are B (MMA N = 16), the fp32 accumulator lives in TMEM.
//    One kernel serves every M = 1..16, so a row's sum does not depend on the number of rows.
//  * TMA streams 128-row weight tiles (16 KB per stage, 128-byte swizzle, L2 evict-first) and the
//    matching activation tile (rows beyond M zero-filled by TMA) into a shared-memory ring.
//  * bf16 weights feed the MMA from shared memory. int8 weights are widened to bf16 by four converter
//    warps (exact: byte permute into 2^23 + u, one subtract, upper half) and stored into TMEM, from where
//    the MMA reads its A operand; the widened weights never go back through shared memory.
//  * Two work partitions, chosen from (N, K) only (never from M):
//     - stream-K (many tiles): a persistent grid of one CTA per SM; CTA c owns the contiguous unit range
//       [c U / P, (c + 1) U / P) of the U = tiles x k-blocks units, so every SM streams the same number
//       of bytes. A tile split between CTAs is finished by the CTA that arrives last (atomic counter per
//       tile, reset by that CTA), adding the partials in CTA order: deterministic, and no CTA waits.
//     - cluster split-K (few tiles): the S CTAs of a thread-block cluster split one tile's K range and
//       add their partials through distributed shared memory, in rank order.
//  * Warp roles: warp 0 issues TMA, warp 1 issues tcgen05.mma (and owns the TMEM allocation), the
//    epilogue warps drain TMEM (two accumulator buffers, so draining overlaps the next tile's MMAs).
//  * Programmatic dependent launch: every CTA lets the next kernel in the stream launch at once, and
//    issues its first weight tiles before griddepcontrol.wait (weights are not produced by the
//    preceding kernel; the activations and every global write come after the wait).
//  * Every mbarrier wait is bounded; a timeout sets the device error word, the CTA drains its copies
//    in flight, frees TMEM and returns.
#include <cudaTypedefs.h>

#include "skinny_internal.h"
#include "sm100.cuh"

namespace bp {
namespace {

constexpr int kBM = 128;  // weight rows per tile (MMA M)
constexpr int kNP = 16;   // activation rows per launch (MMA N)
constexpr int kEpiThreads = 128;

template <bool kInt8>
struct TcTraits;
template <>
struct TcTraits<false> {                   // bf16 weights
  static constexpr int BK = 64;            // K elements per stage (one 128-byte swizzle row)
  static constexpr int STAGES = 6;
  static constexpr int A_BYTES = kBM * BK * 2;
  static constexpr int B_BYTES = kNP * BK * 2;
  static constexpr int THREADS = 192;      // TMA, MMA, 4 epilogue warps
  static constexpr int EPI_WARP0 = 2;
  static constexpr int A_SLOTS = 1;        // unused
  static constexpr uint32_t TMEM_COLS = 32;  // two 16-column accumulators
};
template <>
struct TcTraits<true> {                    // int8 weights
  static constexpr int BK = 128;           // K elements per stage (128 bytes of int8 per row)
  static constexpr int STAGES = 5;
  static constexpr int A_BYTES = kBM * BK;
  static constexpr int B_BYTES = kNP * BK * 2;  // two 64-wide activation boxes
  static constexpr int THREADS = 320;      // TMA, MMA, 4 converter warps, 4 epilogue warps
  static constexpr int EPI_WARP0 = 6;
  static constexpr int A_SLOTS = 3;        // widened A tiles in TMEM: 64 columns each at 64, 128, 192
  static constexpr uint32_t TMEM_COLS = 256;
};

struct TcArgs {
  void* y;
  long long ldy;
  int y_f32;
  const __nv_bfloat16* scale;  // int8: [N] per-row scale; bf16: NULL
  int M, N, K;
  int tiles, kblocks;
  long long units;
  int P;            // CTAs
  int S;            // cluster mode: CTAs per tile; 0: stream-K mode
  int* counters;    // stream-K: [tiles], zero between launches
  float* partials;  // stream-K: [P][2][kNP][kBM]
};

template <bool kInt8>
struct __align__(1024) TcSmem {
  using Tr = TcTraits<kInt8>;
  uint8_t a[Tr::STAGES][Tr::A_BYTES];
  uint8_t b[Tr::STAGES][Tr::B_BYTES];
  uint64_t full[Tr::STAGES];
  uint64_t empty[Tr::STAGES];
  uint64_t tfull[2];
  uint64_t tempty[2];
  uint64_t afull[Tr::A_SLOTS];
  uint64_t aempty[Tr::A_SLOTS];
  uint64_t mma_done;
  uint32_t tmem_base;
  int abort;
  int last_flag;
};

template <bool kInt8>
constexpr size_t smem_bytes() {
  return sizeof(TcSmem<kInt8>) + 1024;  // + slack to align the base to 1024 bytes
}

__host__ __device__ __forceinline__ long long unit_start(int c, long long U, int P) {
  return static_cast<long long>(c) * U / P;
}
// The CTA whose range holds unit u: the largest c with unit_start(c) <= u.
__host__ __device__ __forceinline__ int unit_owner(long long u, long long U, int P) {
  return static_cast<int>(((u + 1) * P - 1) / U);
}

// Waits that ignore `abort`: used only to drain this CTA's own asynchronous work before it exits.
__device__ __forceinline__ void mbar_wait_drain(uint64_t* bar, uint32_t parity) {
  const unsigned long long t0 = globaltimer();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer() - t0 > kWaitLimitNs) {
      atomicOr(&g_bp_device_errors, BP_DEVERR_TIMEOUT);
      return;
    }
  }
}

__device__ __forceinline__ void store_value(const TcArgs& a, int m, int row, float v) {
  if (a.scale != nullptr) v *= __bfloat162float(a.scale[row]);
  if (a.y_f32)
    static_cast<float*>(a.y)[m * a.ldy + row] = v;
  else
    static_cast<__nv_bfloat16*>(a.y)[m * a.ldy + row] = __float2bfloat16_rn(v);
}

__device__ __forceinline__ void store_rows(const TcArgs& a, int row, const float (&v)[kNP]) {
  if (row >= a.N) return;
#pragma unroll
  for (int m = 0; m < kNP; ++m)
    if (m < a.M) store_value(a, m, row, v[m]);
}

// 16 signed bytes (one 16-byte chunk of an int8 weight row) -> 8 exact bf16x2 words.
__device__ __forceinline__ void widen_int8x16(const uint4& v, uint32_t* out) {
  const uint32_t words[4] = {v.x ^ 0x80808080u, v.y ^ 0x80808080u, v.z ^ 0x80808080u, v.w ^ 0x80808080u};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      // q = (2^23 + u) - (2^23 + 128) exactly in fp32; |q| <= 127 has at most 7 significant bits, so the
      // upper half of its fp32 pattern is exactly bf16(q)
      const float lo = __uint_as_float(__byte_perm(words[j], 0x4B000000u, 0x7540u | (2 * h))) - 8388736.0f;
      const float hi = __uint_as_float(__byte_perm(words[j], 0x4B000000u, 0x7540u | (2 * h + 1))) - 8388736.0f;
      out[2 * j + h] = __byte_perm(__float_as_uint(lo), __float_as_uint(hi), 0x7632u);
    }
  }
}

__device__ __forceinline__ void tmem_st_32x32b_x64(uint32_t taddr, const uint32_t (&r)[64]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x64.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32, %33, %34, %35, %36, "
      "%37, %38, %39, %40, %41, %42, %43, %44, %45, %46, %47, %48, %49, %50, %51, %52, %53, %54, %55, %56, %57, %58, "
      "%59, %60, %61, %62, %63, %64};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
      "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
      "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31]), "r"(r[32]), "r"(r[33]), "r"(r[34]), "r"(r[35]), "r"(r[36]),
      "r"(r[37]), "r"(r[38]), "r"(r[39]), "r"(r[40]), "r"(r[41]), "r"(r[42]), "r"(r[43]), "r"(r[44]), "r"(r[45]),
      "r"(r[46]), "r"(r[47]), "r"(r[48]), "r"(r[49]), "r"(r[50]), "r"(r[51]), "r"(r[52]), "r"(r[53]), "r"(r[54]),
      "r"(r[55]), "r"(r[56]), "r"(r[57]), "r"(r[58]), "r"(r[59]), "r"(r[60]), "r"(r[61]), "r"(r[62]), "r"(r[63])
      : "memory");
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// D[tmem] (+)= A[tmem] . B[smem]^T (A read from tensor memory), bf16 inputs, fp32 accumulator.
__device__ __forceinline__ void umma_f16_tmem_a(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                                uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}"
      ::"r"(d_tmem), "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// kCluster = false: stream-K over (tile, k-block) units, split tiles finished through the workspace.
// kCluster = true: grid = tiles x S, the S CTAs of a cluster split one tile's K range evenly and add
// their partials through distributed shared memory (used when there are few tiles).
template <bool kInt8, bool kCluster>
__global__ void __launch_bounds__(TcTraits<kInt8>::THREADS, 2)
    skinny_tc_kernel(const __grid_constant__ CUtensorMap tw, const __grid_constant__ CUtensorMap tx, const TcArgs a) {
  using Tr = TcTraits<kInt8>;
  constexpr int STAGES = Tr::STAGES, BK = Tr::BK;
  extern __shared__ uint8_t smem_raw[];
  TcSmem<kInt8>& s =
      *reinterpret_cast<TcSmem<kInt8>*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
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
    for (int i = 0; i < STAGES; ++i) {
      mbar_init(&s.full[i], 1);
      mbar_init(&s.empty[i], kInt8 ? 1 + 128 : 1);  // int8: the MMA's commit + the 128 converter threads
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&s.tfull[b], 1);
      mbar_init(&s.tempty[b], kEpiThreads);
    }
    for (int j = 0; j < Tr::A_SLOTS; ++j) {
      mbar_init(&s.afull[j], 128);
      mbar_init(&s.aempty[j], 1);
    }
    mbar_init(&s.mma_done, 1);
    s.abort = 0;
    s.last_flag = 0;
    mbar_fence_init();
    tma_prefetch_desc(&tw);
    tma_prefetch_desc(&tx);
  }
  if (warp == 1) {
    tmem_alloc(&s.tmem_base, Tr::TMEM_COLS);
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
      // ---- TMA producer ----
      const uint64_t pol = l2_evict_first_policy();
      const int npre = n_units < STAGES ? n_units : STAGES;
      for (int i = 0; i < npre; ++i) {  // weights only: they do not depend on the previous kernel
        const long long u = u0 + i;
        const int t = static_cast<int>(u / KB), kb = static_cast<int>(u % KB);
        mbar_arrive_expect_tx(&s.full[i], Tr::A_BYTES + Tr::B_BYTES);
        tma_load_2d_hint(s.a[i], &tw, &s.full[i], kb * BK, t * kBM, pol);
      }
      pdl_wait_prior_grids();
      auto load_x = [&](int st, int kb) {
        tma_load_2d(s.b[st], &tx, &s.full[st], kb * BK, 0);
        if constexpr (kInt8) tma_load_2d(s.b[st] + Tr::B_BYTES / 2, &tx, &s.full[st], kb * BK + 64, 0);
      };
      for (int i = 0; i < npre; ++i) load_x(i, static_cast<int>((u0 + i) % KB));
      int issued = npre;
      for (int i = npre; i < n_units; ++i) {
        const int st = i % STAGES;
        if (!mbar_wait(&s.empty[st], static_cast<uint32_t>((i / STAGES) + 1) & 1u, abort)) break;
        const long long u = u0 + i;
        const int t = static_cast<int>(u / KB), kb = static_cast<int>(u % KB);
        mbar_arrive_expect_tx(&s.full[st], Tr::A_BYTES + Tr::B_BYTES);
        tma_load_2d_hint(s.a[st], &tw, &s.full[st], kb * BK, t * kBM, pol);
        load_x(st, kb);
        issued = i + 1;
      }
      // drain: the last copy issued into each stage has landed
      for (int st = 0; st < STAGES && st < issued; ++st) {
        const int i_last = st + STAGES * ((issued - 1 - st) / STAGES);
        mbar_wait_drain(&s.full[st], static_cast<uint32_t>(i_last / STAGES) & 1u);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---- MMA issuer ----
      constexpr uint32_t idesc = umma_idesc_bf16(kBM, kNP);
      int i = 0, it = 0;
      bool ok = true;
      for (int t = t_first; t <= t_last && ok; ++t, ++it) {
        const long long lo = u0 > static_cast<long long>(t) * KB ? u0 : static_cast<long long>(t) * KB;
        const long long hi = u1 < static_cast<long long>(t + 1) * KB ? u1 : static_cast<long long>(t + 1) * KB;
        const int buf = it & 1;
        if (!mbar_wait(&s.tempty[buf], static_cast<uint32_t>((it >> 1) + 1) & 1u, abort)) break;
        tc_fence_after_sync();
        const uint32_t dacc = tmem + static_cast<uint32_t>(buf * kNP);
        for (long long u = lo; u < hi; ++u, ++i) {
          const int st = i % STAGES;
          if (!mbar_wait(&s.full[st], static_cast<uint32_t>(i / STAGES) & 1u, abort)) {
            ok = false;
            break;
          }
          const uint32_t bb = smem_addr(s.b[st]);
          if constexpr (kInt8) {
            const int slot = i % Tr::A_SLOTS;
            if (!mbar_wait(&s.afull[slot], static_cast<uint32_t>(i / Tr::A_SLOTS) & 1u, abort)) {
              ok = false;
              break;
            }
            tc_fence_after_sync();
            const uint32_t at = tmem + 64u * static_cast<uint32_t>(1 + slot);
#pragma unroll
            for (int kk = 0; kk < BK / 16; ++kk)
              umma_f16_tmem_a(dacc, at + 8u * kk, umma_desc_sw128(bb + (kk >> 2) * (Tr::B_BYTES / 2) + 32 * (kk & 3)),
                              idesc, (u > lo || kk > 0) ? 1u : 0u);
            umma_commit(&s.aempty[slot]);  // the widened tile's TMEM slot is free once these MMAs are done
          } else {
            tc_fence_after_sync();
            const uint32_t ab = smem_addr(s.a[st]);
#pragma unroll
            for (int kk = 0; kk < BK / 16; ++kk)
              umma_f16(dacc, umma_desc_sw128(ab + 32 * kk), umma_desc_sw128(bb + 32 * kk), idesc,
                       (u > lo || kk > 0) ? 1u : 0u);
          }
          umma_commit(&s.empty[st]);  // frees the stage once these MMAs have read it
        }
        if (ok) umma_commit(&s.tfull[buf]);
      }
      umma_commit(&s.mma_done);
      mbar_wait_drain(&s.mma_done, 0);
    }
  } else if (kInt8 && warp < Tr::EPI_WARP0) {
    // ---- int8 converters: shared-memory int8 tile -> exact bf16 -> TMEM (the MMA's A operand) ----
    const int q = warp & 3;  // TMEM lane quadrant this warp may access
    const int r = 32 * q + lane;
    for (int i = 0; i < n_units; ++i) {
      const int st = i % STAGES, slot = i % Tr::A_SLOTS;
      bool ok = mbar_wait(&s.aempty[slot], static_cast<uint32_t>((i / Tr::A_SLOTS) + 1) & 1u, abort);
      ok = ok && mbar_wait(&s.full[st], static_cast<uint32_t>(i / STAGES) & 1u, abort);
      if (!__all_sync(0xffffffffu, ok)) break;  // the TMEM store below is warp-collective
      tc_fence_after_sync();
      uint32_t w[64];
      const uint8_t* row = s.a[st] + r * 128;
#pragma unroll
      for (int j = 0; j < 8; ++j) {  // 16-byte chunk j of the row sits at chunk j ^ (row & 7) (128-byte swizzle)
        const uint4 v = *reinterpret_cast<const uint4*>(row + 16 * (j ^ (r & 7)));
        widen_int8x16(v, w + 8 * j);
      }
      tmem_st_32x32b_x64(tmem + (static_cast<uint32_t>(32 * q) << 16) + 64u * static_cast<uint32_t>(1 + slot), w);
      tc_fence_before_sync();
      mbar_arrive(&s.afull[slot]);
      mbar_arrive(&s.empty[st]);  // this thread is done with the int8 tile in shared memory
    }
  } else {
    // ---- epilogue: TMEM -> registers -> y (or a stream-K / cluster partial) ----
    pdl_wait_prior_grids();
    const int q = warp & 3;  // TMEM lane quadrant this warp may access
    const int r = 32 * q + lane;
    const int et = threadIdx.x - 32 * Tr::EPI_WARP0;
    int it = 0;
    for (int t = t_first; t <= t_last; ++t, ++it) {
      const int buf = it & 1;
      const bool ok = mbar_wait(&s.tfull[buf], static_cast<uint32_t>(it >> 1) & 1u, abort);
      __syncwarp();
      if (named_barrier_or(1, kEpiThreads, !ok)) break;  // all epilogue threads take the same decision
      tc_fence_after_sync();
      float acc[kNP];
      tmem_ld_32x32b_x16(tmem + (static_cast<uint32_t>(32 * q) << 16) + static_cast<uint32_t>(buf * kNP), acc);
      tc_fence_before_sync();
      mbar_arrive(&s.tempty[buf]);
      if constexpr (kCluster) {
        // one tile per CTA: the partial goes to this CTA's shared memory (stage 0 is free: every MMA and
        // converter that read it has finished) for the cluster reduction below
        float* red = reinterpret_cast<float*>(s.a[0]);
#pragma unroll
        for (int m = 0; m < kNP; ++m)
          if (m < a.M) red[m * kBM + r] = acc[m];
        continue;
      }
      const int row = t * kBM + r;
      const int c_lo = unit_owner(static_cast<long long>(t) * KB, U, a.P);
      const int c_hi = unit_owner(static_cast<long long>(t + 1) * KB - 1, U, a.P);
      if (c_lo == c_hi) {
        store_rows(a, row, acc);
        continue;
      }
      const int slot = (t == t_first) ? 0 : 1;
      float* mine = a.partials + static_cast<size_t>(c * 2 + slot) * kNP * kBM;
#pragma unroll
      for (int m = 0; m < kNP; ++m)
        if (m < a.M) mine[m * kBM + r] = acc[m];  // only the live activation rows travel
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
      if (s.last_flag) {
        float v[kNP];
#pragma unroll
        for (int m = 0; m < kNP; ++m) v[m] = 0.0f;
        // fixed order c_lo..c_hi (the sum does not depend on arrival order); four contributors' loads
        // are in flight at once
        int cc = c_lo;
        for (; cc + 3 <= c_hi; cc += 4) {
          float t4[4][kNP];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int cj = cc + j;
            const int cslot = (t == static_cast<int>(unit_start(cj, U, a.P) / KB)) ? 0 : 1;
            const float* p = a.partials + static_cast<size_t>(cj * 2 + cslot) * kNP * kBM;
#pragma unroll
            for (int m = 0; m < kNP; ++m) t4[j][m] = m < a.M ? __ldcg(p + m * kBM + r) : 0.0f;
          }
#pragma unroll
          for (int j = 0; j < 4; ++j)
#pragma unroll
            for (int m = 0; m < kNP; ++m) v[m] += t4[j][m];
        }
        for (; cc <= c_hi; ++cc) {
          const int cslot = (t == static_cast<int>(unit_start(cc, U, a.P) / KB)) ? 0 : 1;
          const float* p = a.partials + static_cast<size_t>(cc * 2 + cslot) * kNP * kBM;
#pragma unroll
          for (int m = 0; m < kNP; ++m)
            if (m < a.M) v[m] += __ldcg(p + m * kBM + r);
        }
        store_rows(a, row, v);
      }
    }
  }

  if constexpr (kCluster) {
    // Split-K through distributed shared memory: CTA `rank` finishes rows [rank R, rank R + R) of the
    // tile, adding the S partials in rank order (deterministic), then stores them.
    cluster_sync_unaligned();  // every CTA's partial is in its shared memory
    const int S = a.S;
    const int R = (kBM + S - 1) / S;
    const int r0 = rank * R;
    const int nrows = r0 >= kBM ? 0 : (r0 + R <= kBM ? R : kBM - r0);
    const int t = static_cast<int>(cluster_id_x());
    const uint32_t red = smem_addr(s.a[0]);
    if (!*abort) {
      for (int item = threadIdx.x; item < nrows * a.M; item += Tr::THREADS) {
        const int m = item / nrows, lr = item - m * nrows;
        const int rr = r0 + lr;
        const uint32_t off = red + static_cast<uint32_t>((m * kBM + rr) * 4);
        float part[16];
#pragma unroll
        for (int qq = 0; qq < 16; ++qq) part[qq] = qq < S ? ld_shared_cluster_f32(mapa_shared(off, qq)) : 0.0f;
        float v = 0.0f;
#pragma unroll
        for (int qq = 0; qq < 16; ++qq)
          if (qq < S) v += part[qq];
        const int row = t * kBM + rr;
        if (row < a.N) store_value(a, m, row, v);
      }
    }
    cluster_sync_unaligned();  // peers have finished reading this CTA's shared memory
  }

  tc_fence_before_sync();
  cta_barrier_unaligned();  // lanes 1-31 of warps 0 and 1 arrive while lane 0 still runs its loop
  if (warp == 1) {
    __syncwarp();  // lane 0 ran the MMA loop alone: reconverge before the warp-wide dealloc
    tc_fence_after_sync();
    tmem_dealloc(tmem, Tr::TMEM_COLS);
  }
}

// ---- host side ---------------------------------------------------------------------------------

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (fn == nullptr) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

int encode_2d(CUtensorMap* map, CUtensorMapDataType dtype, const void* base, uint64_t inner, uint64_t outer,
              uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer, CUtensorMapL2promotion promo) {
  auto fn = encode_fn();
  if (fn == nullptr) return fail(BP_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, dtype, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, promo, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(BP_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", static_cast<int>(r));
  return BP_OK;
}

int tc_sm_count() {
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

template <bool kInt8, bool kCluster>
int ensure_attrs() {
  static bool done[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && done[dev]) return BP_OK;
  cudaError_t e = cudaFuncSetAttribute(skinny_tc_kernel<kInt8, kCluster>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem_bytes<kInt8>()));
  if (e != cudaSuccess)
    return fail(BP_ERR_CUDA, "cudaFuncSetAttribute(smem %zu): %s", smem_bytes<kInt8>(), cudaGetErrorString(e));
  if (dev >= 0 && dev < 64) done[dev] = true;
  return BP_OK;
}

bool pdl_enabled() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("BP_DISABLE_PDL");
    v = (e != nullptr && e[0] == '1') ? 0 : 1;
  }
  return v == 1;
}

constexpr int kMaxClusterSplit = 8;  // portable cluster size

// Work partition; depends on (N, K, weight type) and the SM count only, never on M.
struct Partition {
  int tiles, kblocks, P, S;  // S > 0: cluster mode with S CTAs per tile; S == 0: stream-K over P CTAs
  long long units;
};

Partition partition(int N, int K, int bk) {
  Partition p;
  p.tiles = (N + kBM - 1) / kBM;
  p.kblocks = (K + bk - 1) / bk;
  p.units = static_cast<long long>(p.tiles) * p.kblocks;
  const int sms = tc_sm_count();
  if (2 * p.tiles <= sms) {
    // few tiles: split each tile's K range over a cluster of S CTAs (no workspace, no global fix-up)
    int S = sms / p.tiles;
    if (S > kMaxClusterSplit) S = kMaxClusterSplit;
    if (S > p.kblocks) S = p.kblocks;
    p.S = S < 1 ? 1 : S;
    p.P = p.tiles * p.S;
  } else {
    p.S = 0;
    p.P = static_cast<int>(p.units < sms ? p.units : sms);
  }
  return p;
}

// The workspace layout is the same for every shape: kMaxTiles tile counters, then the partials. (A
// layout that depended on the tile count would let one shape's partials land on another shape's
// counters, which must stay zero between launches.)
constexpr int kMaxTiles = 8192;  // N up to 1,048,576 rows
constexpr size_t kCountersBytes = static_cast<size_t>(kMaxTiles) * 4;

template <bool kInt8, bool kCluster>
cudaError_t launch_kernel(cudaLaunchConfig_t* cfg, const CUtensorMap& tw, const CUtensorMap& tx, const TcArgs& a) {
  return cudaLaunchKernelEx(cfg, skinny_tc_kernel<kInt8, kCluster>, tw, tx, a);
}

}  // namespace

size_t skinny_tc_workspace_bytes(int N, int K, bool int8) {
  if (N <= 0 || K <= 0) return 0;
  const Partition p = partition(N, K, int8 ? TcTraits<true>::BK : TcTraits<false>::BK);
  if (p.S > 0) return 0;  // cluster mode needs no workspace
  return kCountersBytes + static_cast<size_t>(p.P) * 2 * kNP * kBM * sizeof(float);
}

bool skinny_tc_supported(const void* x, long long ldx, const void* w, int M, int N, int K, bool int8) {
  const bool al = (reinterpret_cast<uintptr_t>(x) & 15u) == 0 && (reinterpret_cast<uintptr_t>(w) & 15u) == 0;
  const bool k_ok = int8 ? (K >= 128 && K % 128 == 0) : (K >= 8 && K % 8 == 0);
  return al && k_ok && M >= 1 && M <= kNP && N >= 1 && (N + kBM - 1) / kBM <= kMaxTiles && ldx % 8 == 0;
}

int launch_skinny_tc(const void* x, long long ldx, const void* w, const void* w_scale, void* y, long long ldy, int y_f32,
                     int M, int N, int K, bool int8, void* ws, size_t ws_bytes, cudaStream_t stream) {
  const int bk = int8 ? TcTraits<true>::BK : TcTraits<false>::BK;
  const Partition p = partition(N, K, bk);
  const size_t need = skinny_tc_workspace_bytes(N, K, int8);
  if (need > 0 && (ws == nullptr || ws_bytes < need))
    return fail(BP_ERR_INVALID_ARGUMENT, "the tensor-core path needs a zero-initialised workspace of %zu bytes (got %zu)",
                need, ws_bytes);
  if (need > 0 && (reinterpret_cast<uintptr_t>(ws) & 255u) != 0)
    return fail(BP_ERR_MISALIGNED, "workspace must be 256-byte aligned");
  int st;
  if (int8)
    st = p.S > 0 ? ensure_attrs<true, true>() : ensure_attrs<true, false>();
  else
    st = p.S > 0 ? ensure_attrs<false, true>() : ensure_attrs<false, false>();
  if (st != BP_OK) return st;
  CUtensorMap tw, tx;
  if (int8)
    st = encode_2d(&tw, CU_TENSOR_MAP_DATA_TYPE_UINT8, w, static_cast<uint64_t>(K), static_cast<uint64_t>(N),
                   static_cast<uint64_t>(K), 128, kBM, CU_TENSOR_MAP_L2_PROMOTION_L2_256B);
  else
    st = encode_2d(&tw, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, w, static_cast<uint64_t>(K), static_cast<uint64_t>(N),
                   static_cast<uint64_t>(K) * 2, 64, kBM, CU_TENSOR_MAP_L2_PROMOTION_L2_256B);
  if (st != BP_OK) return st;
  st = encode_2d(&tx, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, x, static_cast<uint64_t>(K), static_cast<uint64_t>(M),
                 static_cast<uint64_t>(ldx) * 2, 64, kNP, CU_TENSOR_MAP_L2_PROMOTION_L2_128B);
  if (st != BP_OK) return st;

  TcArgs a;
  a.y = y;
  a.ldy = ldy;
  a.y_f32 = y_f32;
  a.scale = int8 ? static_cast<const __nv_bfloat16*>(w_scale) : nullptr;
  a.M = M;
  a.N = N;
  a.K = K;
  a.tiles = p.tiles;
  a.kblocks = p.kblocks;
  a.units = p.units;
  a.P = p.P;
  a.S = p.S;
  a.counters = need > 0 ? static_cast<int*>(ws) : nullptr;
  a.partials = need > 0 ? reinterpret_cast<float*>(static_cast<char*>(ws) + kCountersBytes) : nullptr;

  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.P, 1, 1);
  cfg.blockDim = dim3(int8 ? TcTraits<true>::THREADS : TcTraits<false>::THREADS, 1, 1);
  cfg.dynamicSmemBytes = int8 ? smem_bytes<true>() : smem_bytes<false>();
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  int na = 0;
  if (pdl_enabled()) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  if (p.S > 0) {
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = p.S;
    attr[na].val.clusterDim.y = 1;
    attr[na].val.clusterDim.z = 1;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  cudaError_t e;
  if (int8)
    e = p.S > 0 ? launch_kernel<true, true>(&cfg, tw, tx, a) : launch_kernel<true, false>(&cfg, tw, tx, a);
  else
    e = p.S > 0 ? launch_kernel<false, true>(&cfg, tw, tx, a) : launch_kernel<false, false>(&cfg, tw, tx, a);
  if (e != cudaSuccess)
    return fail(BP_ERR_CUDA, "tensor-core skinny launch (%s M=%d N=%d K=%d P=%d S=%d): %s", int8 ? "int8" : "bf16", M, N,
                K, p.P, p.S, cudaGetErrorString(e));
  return BP_OK;
}

// ---- entry point for callers that cannot allocate device memory -----------------------------------
//
// Some callers have no way to allocate device memory for the stream-K scratch: code that runs while a
// stream is being captured into a CUDA graph in global capture mode (cudaMalloc is refused there), and
// host applications that hand out all device memory from their own pre-reserved pool and give plugins
// no allocator. For them, the scratch of the tensor-core path lives in this fixed array instead of a
// caller-provided workspace. It is part of the module, so every GPU that loads the library holds it
// (2.6 MB) until the process exits. Limits: at most kStaticMaxCtas streaming multiprocessors (B200 has
// 148) and N <= kMaxTiles * 128 rows; larger problems are rejected with BP_ERR_UNSUPPORTED.
constexpr int kStaticMaxCtas = 160;
constexpr size_t kStaticScratchBytes =
    kCountersBytes + static_cast<size_t>(kStaticMaxCtas) * 2 * kNP * kBM * sizeof(float);
static __device__ __align__(256) unsigned char g_static_scratch[kStaticScratchBytes];

// Device address of g_static_scratch on the current device (host code must not pass the symbol itself:
// on the host it is only a stand-in). Looked up once per device.
static int static_scratch_ptr(void** out) {
  static void* ptrs[64] = {nullptr};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(BP_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= 64) return fail(BP_ERR_UNSUPPORTED, "device index %d out of range", dev);
  if (ptrs[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_static_scratch);
    if (e != cudaSuccess || p == nullptr)
      return fail(BP_ERR_CUDA, "cudaGetSymbolAddress(static scratch): %s", cudaGetErrorString(e));
    ptrs[dev] = p;
  }
  *out = ptrs[dev];
  return BP_OK;
}

}  // namespace bp

extern "C" int bp_skinny_mm_static_scratch(const void* x, long long ldx, const void* w, int w_dtype,
                                           const void* w_scale, void* y, long long ldy, int y_dtype, int M, int N,
                                           int K, void* stream) {
  using namespace bp;
  clear_error();
  if (M > 0 && N > 0 && K > 0 && (w_dtype == BP_DTYPE_BF16 || w_dtype == BP_DTYPE_INT8)) {
    int st = require_sm100();
    if (st != BP_OK) return st;
    const size_t need = skinny_tc_workspace_bytes(N, K, w_dtype == BP_DTYPE_INT8);
    if ((N + kBM - 1) / kBM > kMaxTiles || need > kStaticScratchBytes)
      return fail(BP_ERR_UNSUPPORTED,
                  "N=%d K=%d needs %zu bytes of scratch; the static scratch holds %zu (N <= %d rows, <= %d SMs)", N, K,
                  need, kStaticScratchBytes, kMaxTiles * kBM, kStaticMaxCtas);
    if (need > 0) {
      void* scratch = nullptr;
      st = static_scratch_ptr(&scratch);
      if (st != BP_OK) return st;
      // The tile counters must start at zero. Every call leaves them at zero, but a call that stopped
      // early (device error) would not, so they are cleared on the stream before each call.
      const size_t tiles = static_cast<size_t>((N + kBM - 1) / kBM);
      cudaError_t e = cudaMemsetAsync(scratch, 0, tiles * 4, static_cast<cudaStream_t>(stream));
      if (e != cudaSuccess) return fail(BP_ERR_CUDA, "clearing the static scratch counters: %s", cudaGetErrorString(e));
      return bp_skinny_mm(x, ldx, w, w_dtype, w_scale, y, ldy, y_dtype, M, N, K, scratch, kStaticScratchBytes, stream);
    }
  }
  return bp_skinny_mm(x, ldx, w, w_dtype, w_scale, y, ldy, y_dtype, M, N, K, nullptr, 0, stream);
}

namespace bp {

unsigned int read_and_clear_device_errors() {
  unsigned int v = 0, zero = 0;
  cudaMemcpyFromSymbol(&v, g_bp_device_errors, sizeof(v));
  cudaMemcpyToSymbol(g_bp_device_errors, &zero, sizeof(zero));
  return v;
}

}  // namespace bp
