// Tensor-core skinny linear with bf16 weights: y[M, N] = x[M, K] . W[N, K]^T for M <= 16 rows per launch.
// (int8 weights: skinny_i8.cu.)
//
// Reference: byteprof/optim/skinny.py:35-80 (_skinny_kernel MODE 0: one program per BN weight rows,
// swap-AB tl.dot with the weight tile as the MMA's M operand and the few activation rows as N) and
// skinny.py:83-90, 111-129 (split-K through an fp32 workspace and a second reduce kernel).
//
// B200 design:
//  * Swap-AB on the 5th-generation tensor cores: a 128-row weight tile is the A operand (MMA M = 128),
//    the activation rows padded to 16 are B (MMA N = 16), the fp32 accumulator lives in TMEM.
//    One kernel serves every M = 1..16, so a row's sum does not depend on the number of rows. (An MMA
//    costs about the same for N = 16 as for N = 128, but four bf16 MMAs per 16 KB stage still run far
//    faster than HBM delivers the stage.)
//  * TMA streams 128-row weight tiles (16 KB per stage, 128-byte swizzle, L2 evict-first) and the
//    matching activation tile (rows beyond M zero-filled by TMA) into a shared-memory ring.
//  * Two work partitions, chosen from (N, K) only (never from M):
//     - stream-K (many tiles): a persistent grid of two CTAs per SM; CTA c owns the contiguous unit range
//       [c U / P, (c + 1) U / P) of the U = tiles x k-blocks units, so every SM streams the same number
//       of bytes. A tile split between CTAs is finished by the CTA that arrives last (atomic counter per
//       tile, reset by that CTA), adding the partials in CTA order: deterministic, and no CTA waits.
//     - cluster split-K (few tiles): the S CTAs of a thread-block cluster split one tile's K range; each
//       stores its partial of every row into a slot of the CTA owning that row (distributed shared
//       memory), and after one cluster barrier the owner adds the slots in rank order.
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
constexpr int kBK = 64;   // K elements per stage (one 128-byte swizzle row)
constexpr int kMaxClusterSplit = 8;  // portable cluster size
constexpr int kABytes = kBM * kBK * 2;
constexpr int kBBytes = kNP * kBK * 2;
constexpr int kThreads = 192;  // TMA, MMA, 4 epilogue warps
constexpr int kEpiWarp0 = 2;
constexpr uint32_t kTmemCols = 32;  // two 16-column accumulators
constexpr int kEpiBatch = 4;        // stream-K partials loaded at once by the finishing CTA

struct TcArgs {
  void* y;
  long long ldy;
  int y_f32;
  int M, N, K;
  int tiles, kblocks;
  long long units;
  int P;            // CTAs
  int S;            // cluster mode: CTAs per tile; 0: stream-K mode
  int* counters;    // stream-K: [tiles], zero between launches
  float* partials;  // stream-K: [P][2][kNP][kBM]
};

// Stream-K: a 6-stage ring. Cluster split-K: 5 stages and the slots where the cluster's CTAs store their
// partials of this CTA's rows ([source rank][activation row][row of this CTA's share]), so that two CTAs
// still fit per SM.
template <bool kCluster>
struct TcCfg {
  static constexpr int kStages = kCluster ? 5 : 6;
  static constexpr int kRedElems = kCluster ? kNP * (kBM + kMaxClusterSplit) : 4;
};

template <bool kCluster>
struct __align__(1024) TcSmem {
  uint8_t a[TcCfg<kCluster>::kStages][kABytes];
  uint8_t b[TcCfg<kCluster>::kStages][kBBytes];
  float red[TcCfg<kCluster>::kRedElems];
  uint64_t full[TcCfg<kCluster>::kStages];
  uint64_t empty[TcCfg<kCluster>::kStages];
  uint64_t tfull[2];
  uint64_t tempty[2];
  uint64_t mma_done;
  uint32_t tmem_base;
  int abort;
  int last_flag;
};

template <bool kCluster>
constexpr size_t smem_bytes() {
  return sizeof(TcSmem<kCluster>) + 1024;  // + slack to align the base to 1024 bytes
}
// Two CTAs per SM (so that the next kernel's CTAs start under this one's tail): 228 KB per SM, 1 KB of
// it reserved per CTA.
static_assert(smem_bytes<false>() <= 115712 && smem_bytes<true>() <= 115712, "two CTAs per SM must fit");

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

// kCluster = false: stream-K over (tile, k-block) units, split tiles finished through the workspace.
// kCluster = true: grid = tiles x S, the S CTAs of a cluster split one tile's K range evenly and add
// their partials through distributed shared memory (used when there are few tiles).
template <bool kCluster>
__global__ void __launch_bounds__(kThreads, 2)
    skinny_tc_kernel(const __grid_constant__ CUtensorMap tw, const __grid_constant__ CUtensorMap tx, const TcArgs a) {
  constexpr int kStages = TcCfg<kCluster>::kStages;
  extern __shared__ uint8_t smem_raw[];
  TcSmem<kCluster>& s =
      *reinterpret_cast<TcSmem<kCluster>*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
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
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&s.full[i], 1);
      mbar_init(&s.empty[i], 1);
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
    tma_prefetch_desc(&tx);
  }
  if (warp == 1) {
    tmem_alloc(&s.tmem_base, kTmemCols);
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
      const int npre = n_units < kStages ? n_units : kStages;
      for (int i = 0; i < npre; ++i) {  // weights only: they do not depend on the previous kernel
        const long long u = u0 + i;
        const int t = static_cast<int>(u / KB), kb = static_cast<int>(u % KB);
        mbar_arrive_expect_tx(&s.full[i], kABytes + kBBytes);
        tma_load_2d_hint(s.a[i], &tw, &s.full[i], kb * kBK, t * kBM, pol);
      }
      pdl_wait_prior_grids();
      for (int i = 0; i < npre; ++i) tma_load_2d(s.b[i], &tx, &s.full[i], static_cast<int>((u0 + i) % KB) * kBK, 0);
      int issued = npre;
      for (int i = npre; i < n_units; ++i) {
        const int st = i % kStages;
        if (!mbar_wait(&s.empty[st], static_cast<uint32_t>((i / kStages) + 1) & 1u, abort)) break;
        const long long u = u0 + i;
        const int t = static_cast<int>(u / KB), kb = static_cast<int>(u % KB);
        mbar_arrive_expect_tx(&s.full[st], kABytes + kBBytes);
        tma_load_2d_hint(s.a[st], &tw, &s.full[st], kb * kBK, t * kBM, pol);
        tma_load_2d(s.b[st], &tx, &s.full[st], kb * kBK, 0);
        issued = i + 1;
      }
      // drain: the last copy issued into each stage has landed
      for (int st = 0; st < kStages && st < issued; ++st) {
        const int i_last = st + kStages * ((issued - 1 - st) / kStages);
        mbar_wait_drain(&s.full[st], static_cast<uint32_t>(i_last / kStages) & 1u);
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
          const int st = i % kStages;
          if (!mbar_wait(&s.full[st], static_cast<uint32_t>(i / kStages) & 1u, abort)) {
            ok = false;
            break;
          }
          tc_fence_after_sync();
          const uint32_t ab = smem_addr(s.a[st]), bb = smem_addr(s.b[st]);
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk)
            umma_f16(dacc, umma_desc_sw128(ab + 32 * kk), umma_desc_sw128(bb + 32 * kk), idesc,
                     (u > lo || kk > 0) ? 1u : 0u);
          umma_commit(&s.empty[st]);  // frees the stage once these MMAs have read it
        }
        if (ok) umma_commit(&s.tfull[buf]);
      }
      umma_commit(&s.mma_done);
      mbar_wait_drain(&s.mma_done, 0);
    }
  } else {
    // ---- epilogue: TMEM -> registers -> y (or a stream-K / cluster partial) ----
    pdl_wait_prior_grids();
    const int q = warp & 3;  // TMEM lane quadrant this warp may access
    const int r = 32 * q + lane;
    const int et = threadIdx.x - 32 * kEpiWarp0;
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
        // one tile per CTA: row r's partial goes to the slot for this rank in the CTA that owns row r
        const int R = (kBM + a.S - 1) / a.S;
        const int own = r / R;
        const uint32_t dst = mapa_shared(smem_addr(&s.red[rank * kNP * R + (r - own * R)]), static_cast<uint32_t>(own));
#pragma unroll
        for (int m = 0; m < kNP; ++m)
          if (m < a.M)
            asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(dst + static_cast<uint32_t>(m * R * 4)), "f"(acc[m])
                         : "memory");
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
        // fixed order c_lo..c_hi (the sum does not depend on arrival order); kEpiBatch contributors'
        // loads are in flight at once
        int cc = c_lo;
        for (; cc + kEpiBatch - 1 <= c_hi; cc += kEpiBatch) {
          float t4[kEpiBatch][kNP];
#pragma unroll
          for (int j = 0; j < kEpiBatch; ++j) {
            const int cj = cc + j;
            const int cslot = (t == static_cast<int>(unit_start(cj, U, a.P) / KB)) ? 0 : 1;
            const float* p = a.partials + static_cast<size_t>(cj * 2 + cslot) * kNP * kBM;
#pragma unroll
            for (int m = 0; m < kNP; ++m) t4[j][m] = m < a.M ? __ldcg(p + m * kBM + r) : 0.0f;
          }
#pragma unroll
          for (int j = 0; j < kEpiBatch; ++j)
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
    // Split-K through distributed shared memory: every CTA of the cluster has stored its partials of
    // rows [rank R, rank R + R) into this CTA's slots; one barrier, then this CTA adds them in rank order
    // (deterministic) and stores the rows. Nothing reads another CTA's memory after the barrier.
    cluster_sync_unaligned();  // release / acquire: every remote store has landed
    const int S = a.S;
    const int R = (kBM + S - 1) / S;
    const int r0 = rank * R;
    const int nrows = r0 >= kBM ? 0 : (r0 + R <= kBM ? R : kBM - r0);
    const int t = static_cast<int>(cluster_id_x());
    if (!*abort) {
      for (int item = threadIdx.x; item < nrows * a.M; item += kThreads) {
        const int m = item / nrows, lr = item - m * nrows;
        float v = 0.0f;
        for (int src = 0; src < S; ++src) v += s.red[(src * kNP + m) * R + lr];
        const int row = t * kBM + r0 + lr;
        if (row < a.N) store_value(a, m, row, v);
      }
    }
  }

  tc_fence_before_sync();
  cta_teardown_barrier();  // every thread has finished with TMEM before warp 1 frees it
  if (warp == 1) {
    tc_fence_after_sync();
    tmem_dealloc(tmem, kTmemCols);
  }
}

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

template <bool kCluster>
int ensure_attrs() {
  static bool done[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && done[dev]) return BP_OK;
  cudaError_t e = cudaFuncSetAttribute(skinny_tc_kernel<kCluster>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem_bytes<kCluster>()));
  if (e != cudaSuccess)
    return fail(BP_ERR_CUDA, "cudaFuncSetAttribute(smem %zu): %s", smem_bytes<kCluster>(), cudaGetErrorString(e));
  if (dev >= 0 && dev < 64) done[dev] = true;
  return BP_OK;
}

// Work partition; depends on (N, K) and the SM count only, never on M.
struct Partition {
  int tiles, kblocks, P, S;  // S > 0: cluster mode with S CTAs per tile; S == 0: stream-K over P CTAs
  long long units;
};

Partition partition(int N, int K) {
  Partition p;
  p.tiles = (N + kBM - 1) / kBM;
  p.kblocks = (K + kBK - 1) / kBK;
  p.units = static_cast<long long>(p.tiles) * p.kblocks;
  const int sms = tc_sm_count();
  if (2 * p.tiles <= sms) {
    // few tiles: split each tile's K range over a cluster of S CTAs (no workspace, no global fix-up). Two
    // CTAs fit per SM, so S = 2 SMs / tiles: every SM then runs two producers, and a single producer issuing
    // a weight and an activation copy per stage streams well below the SM's share of HBM (measured on
    // 8192 x 2048: 9.9 us with S = 2, 8.5 us with S = 4)
    int S = 2 * sms / p.tiles;
    if (S > kMaxClusterSplit) S = kMaxClusterSplit;
    if (S > p.kblocks) S = p.kblocks;
    p.S = S < 1 ? 1 : S;
    p.P = p.tiles * p.S;
  } else {
    // two CTAs per SM, each with its own 6-stage ring: twice the weight bytes in flight per SM
    p.S = 0;
    p.P = static_cast<int>(p.units < 2 * sms ? p.units : 2 * sms);
  }
  return p;
}

template <bool kCluster>
cudaError_t launch_kernel(cudaLaunchConfig_t* cfg, const CUtensorMap& tw, const CUtensorMap& tx, const TcArgs& a) {
  return cudaLaunchKernelEx(cfg, skinny_tc_kernel<kCluster>, tw, tx, a);
}

size_t skinny_bf16_workspace_bytes(int N, int K) {
  if (N <= 0 || K <= 0) return 0;
  const Partition p = partition(N, K);
  if (p.S > 0) return 0;  // cluster mode needs no workspace
  return kTcCountersBytes + static_cast<size_t>(p.P) * 2 * kNP * kBM * sizeof(float);
}

int launch_skinny_bf16(const void* x, long long ldx, const void* w, void* y, long long ldy, int y_f32, int M, int N,
                       int K, void* ws, size_t ws_bytes, cudaStream_t stream) {
  const Partition p = partition(N, K);
  const size_t need = skinny_bf16_workspace_bytes(N, K);
  if (need > 0 && (ws == nullptr || ws_bytes < need))
    return fail(BP_ERR_INVALID_ARGUMENT, "the tensor-core path needs a zero-initialised workspace of %zu bytes (got %zu)",
                need, ws_bytes);
  if (need > 0 && (reinterpret_cast<uintptr_t>(ws) & 255u) != 0)
    return fail(BP_ERR_MISALIGNED, "workspace must be 256-byte aligned");
  int st = p.S > 0 ? ensure_attrs<true>() : ensure_attrs<false>();
  if (st != BP_OK) return st;
  CUtensorMap tw, tx;
  st = tc_encode_2d(&tw, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, w, static_cast<uint64_t>(K), static_cast<uint64_t>(N),
                    static_cast<uint64_t>(K) * 2, kBK, kBM, CU_TENSOR_MAP_L2_PROMOTION_L2_256B);
  if (st != BP_OK) return st;
  st = tc_encode_2d(&tx, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, x, static_cast<uint64_t>(K), static_cast<uint64_t>(M),
                    static_cast<uint64_t>(ldx) * 2, kBK, kNP, CU_TENSOR_MAP_L2_PROMOTION_L2_128B);
  if (st != BP_OK) return st;

  TcArgs a;
  a.y = y;
  a.ldy = ldy;
  a.y_f32 = y_f32;
  a.M = M;
  a.N = N;
  a.K = K;
  a.tiles = p.tiles;
  a.kblocks = p.kblocks;
  a.units = p.units;
  a.P = p.P;
  a.S = p.S;
  a.counters = need > 0 ? static_cast<int*>(ws) : nullptr;
  a.partials = need > 0 ? reinterpret_cast<float*>(static_cast<char*>(ws) + kTcCountersBytes) : nullptr;

  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.P, 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = p.S > 0 ? smem_bytes<true>() : smem_bytes<false>();
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  int na = 0;
  if (tc_pdl_enabled()) {
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
  const cudaError_t e = p.S > 0 ? launch_kernel<true>(&cfg, tw, tx, a) : launch_kernel<false>(&cfg, tw, tx, a);
  if (e != cudaSuccess)
    return fail(BP_ERR_CUDA, "tensor-core skinny launch (bf16 M=%d N=%d K=%d P=%d S=%d): %s", M, N, K, p.P, p.S,
                cudaGetErrorString(e));
  return BP_OK;
}

}  // namespace

// ---- shared by the bf16 and int8 tensor-core kernels ----------------------------------------------

namespace {

// Encoded tensor maps, cached per host thread: a map depends only on its arguments (address, type, sizes,
// strides, box, swizzle, L2 promotion), so a repeated call with the same arguments reuses the encoding
// instead of paying for it again (eager callers encode up to eight maps per call).
struct MapKey {
  const void* base;
  uint64_t dims[5], strides[4];
  uint32_t box[5];
  int dtype, rank, swizzle, promo;
  bool operator==(const MapKey& o) const {
    if (base != o.base || dtype != o.dtype || rank != o.rank || swizzle != o.swizzle || promo != o.promo) return false;
    for (int i = 0; i < rank; ++i)
      if (dims[i] != o.dims[i] || box[i] != o.box[i] || (i + 1 < rank && strides[i] != o.strides[i])) return false;
    return true;
  }
};
constexpr int kMapCache = 256;
struct MapEntry {
  MapKey key;
  CUtensorMap map;
  bool used;
};
thread_local MapEntry t_maps[kMapCache];

uint32_t map_hash(const MapKey& k) {
  uint64_t h = reinterpret_cast<uintptr_t>(k.base) * 0x9E3779B97F4A7C15ull;
  for (int i = 0; i < k.rank; ++i) h = (h ^ (k.dims[i] * 31 + k.box[i])) * 0x100000001B3ull;
  h ^= static_cast<uint64_t>(k.dtype * 7 + k.swizzle * 131 + k.promo * 1031 + k.rank);
  return static_cast<uint32_t>(h >> 32) % kMapCache;
}

}  // namespace

int tc_encode_2d(CUtensorMap* map, CUtensorMapDataType dtype, const void* base, uint64_t inner, uint64_t outer,
                 uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer, CUtensorMapL2promotion promo) {
  const uint64_t dims[2] = {inner, outer};
  const uint64_t strides[1] = {row_bytes};
  const uint32_t box[2] = {box_inner, box_outer};
  return tc_encode(map, dtype, 2, base, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B, promo);
}

int tc_encode(CUtensorMap* map, CUtensorMapDataType dtype, int rank, const void* base, const uint64_t* dims,
              const uint64_t* strides, const uint32_t* box, CUtensorMapSwizzle swizzle, CUtensorMapL2promotion promo) {
  if (rank < 1 || rank > 5) return fail(BP_ERR_INVALID_ARGUMENT, "tensor map rank %d", rank);
  MapKey key{};
  key.base = base;
  key.dtype = static_cast<int>(dtype);
  key.rank = rank;
  key.swizzle = static_cast<int>(swizzle);
  key.promo = static_cast<int>(promo);
  for (int i = 0; i < rank; ++i) {
    key.dims[i] = dims[i];
    key.box[i] = box[i];
    if (i + 1 < rank) key.strides[i] = strides[i];
  }
  MapEntry& slot = t_maps[map_hash(key)];
  if (slot.used && slot.key == key) {
    *map = slot.map;
    return BP_OK;
  }
  auto fn = encode_fn();
  if (fn == nullptr) return fail(BP_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  cuuint64_t d[5], st[4];
  cuuint32_t b[5], e[5];
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    b[i] = box[i];
    e[i] = 1;
    if (i + 1 < rank) st[i] = strides[i];
  }
  CUresult r = fn(map, dtype, static_cast<cuuint32_t>(rank), const_cast<void*>(base), d, st, b, e,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, promo, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(BP_ERR_CUDA, "cuTensorMapEncodeTiled (rank %d) failed (%d)", rank, static_cast<int>(r));
  slot.key = key;
  slot.map = *map;
  slot.used = true;
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

bool tc_pdl_enabled() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("BP_DISABLE_PDL");
    v = (e != nullptr && e[0] == '1') ? 0 : 1;
  }
  return v == 1;
}

size_t skinny_tc_workspace_bytes(int N, int K, bool int8) {
  return int8 ? skinny_i8_workspace_bytes(N, K) : skinny_bf16_workspace_bytes(N, K);
}

bool skinny_tc_supported(const void* x, long long ldx, const void* w, int M, int N, int K, bool int8) {
  if (int8) return skinny_i8_supported(x, ldx, w, M, N, K);
  const bool al = (reinterpret_cast<uintptr_t>(x) & 15u) == 0 && (reinterpret_cast<uintptr_t>(w) & 15u) == 0;
  return al && K >= 8 && K % 8 == 0 && M >= 1 && M <= kNP && N >= 1 && (N + kBM - 1) / kBM <= kTcMaxTiles &&
         ldx % 8 == 0;
}

int launch_skinny_tc(const void* x, long long ldx, const void* w, const void* w_scale, void* y, long long ldy, int y_f32,
                     int M, int N, int K, bool int8, void* ws, size_t ws_bytes, cudaStream_t stream) {
  if (int8) return launch_skinny_i8(x, ldx, w, w_scale, y, ldy, y_f32, M, N, K, ws, ws_bytes, stream);
  return launch_skinny_bf16(x, ldx, w, y, ldy, y_f32, M, N, K, ws, ws_bytes, stream);
}

// ---- entry point for callers that cannot allocate device memory -----------------------------------
//
// Some callers have no way to allocate device memory for the stream-K scratch: code that runs while a
// stream is being captured into a CUDA graph in global capture mode (cudaMalloc is refused there), and
// host applications that hand out all device memory from their own pre-reserved pool and give plugins
// no allocator. For them, the scratch of the tensor-core paths lives in this fixed array instead of a
// caller-provided workspace. It is part of the module, so every GPU that loads the library holds it
// (11.6 MB: the int8 path's digit matrix and exact int64 partials) until the process exits. Limits: at
// most kStaticMaxCtas streaming multiprocessors (B200 has 148), N <= kTcMaxTiles * 128 rows and, for
// int8 weights, K <= 16384; larger problems are rejected with BP_ERR_UNSUPPORTED.
constexpr int kStaticMaxCtas = 160;
constexpr size_t kStaticPerCta = 2 * 16 * 256 * sizeof(long long);  // the larger of the two paths' per-CTA partials
constexpr size_t kStaticScratchBytes =
    kTcCountersBytes + 1024 + (size_t{64} << 14) + static_cast<size_t>(kStaticMaxCtas) * kStaticPerCta;
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
    // The address is resolved on every such call, whatever the shape, before the size checks: then the
    // first call on a device does the lookup (which may load the module) even when its own shape needs no
    // scratch, and a later call made during stream capture never does.
    void* scratch = nullptr;
    st = static_scratch_ptr(&scratch);
    if (st != BP_OK) return st;
    const size_t need = skinny_tc_workspace_bytes(N, K, w_dtype == BP_DTYPE_INT8);
    if ((N + kBM - 1) / kBM > kTcMaxTiles || need > kStaticScratchBytes)
      return fail(BP_ERR_UNSUPPORTED,
                  "N=%d K=%d needs %zu bytes of scratch; the static scratch holds %zu (N <= %d rows, <= %d SMs)", N, K,
                  need, kStaticScratchBytes, kTcMaxTiles * kBM, kStaticMaxCtas);
    if (need > 0) {
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

BP_DEFINE_DEVICE_ERROR_READER(read_device_errors_tc)

unsigned int read_and_clear_device_errors() {
  return read_device_errors_tc() | read_device_errors_i8() | read_device_errors_i4tc() | read_device_errors_glob() |
         read_device_errors_loc();
}

}  // namespace bp
