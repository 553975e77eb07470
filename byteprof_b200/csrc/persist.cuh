// Machinery shared by the persistent decode kernels (glob_step.cu: the global-model step; loc_step.cu:
// the local encoder and decoder steps): one CTA per SM (cooperative launch), 8 consumer warps and one
// producer warp; the producer streams this CTA's weight rows in 16 KB 1-D bulk copies through a 12-slot
// shared-memory ring; the consumers run the phases of the step, separated by grid barriers on one
// monotonic arrival counter.
//
// Every wait is bounded: a ring wait or a grid barrier that has not completed after kWaitLimitNs sets the
// CTA's abort flag, the grid's abort word and the device error flag; every CTA then leaves once the bulk
// copies it has in flight have landed.
#pragma once

#include "bp_common.cuh"
#include "sm100.cuh"

namespace bp {
namespace persist {

constexpr int kConsumerWarps = 8;
constexpr int kConsumers = kConsumerWarps * 32;  // 256
// Threads of a persistent kernel with P producer warps (the global step uses one, the local steps two).
constexpr int threads_for(int producer_warps) { return kConsumers + 32 * producer_warps; }
constexpr int kSlots = 12;
constexpr int kSlotBytes = 16384;
constexpr unsigned kFull = 0xffffffffu;

// The ring and the CTA's control words; the first member of a kernel's shared-memory struct.
struct Ring {
  alignas(128) uint8_t slot[kSlots][kSlotBytes];
  uint64_t full[kSlots], empty[kSlots];
  int readers[kSlots];  // warps done with each slot
  int issued[kSlots];   // the chunk most recently issued into each slot (-1: none yet)
  int abort;            // this CTA stops (read by the producer's waits)
  int bad;              // consumer-wide result of the last grid barrier
  float red[2][kConsumerWarps];
};

// Thread 0, before the CTA's first barrier.
__device__ __forceinline__ void ring_init(Ring& r) {
  for (int i = 0; i < kSlots; ++i) {
    mbar_init(&r.full[i], 1);
    mbar_init(&r.empty[i], 1);
    r.readers[i] = 0;
    r.issued[i] = -1;
  }
  r.abort = 0;
  r.bad = 0;
  mbar_fence_init();
}

// Rows [r0, r1) of n rows that CTA c of G owns.
// 32-bit unsigned division (c n stays below 2^32 for every row count here: n <= 2^20 rows, g <= 2^11 CTAs;
// 64-bit divisions made each CTA's start-up plan cost about 2 us).
__device__ __forceinline__ void split(int n, int g, int c, int& r0, int& r1) {
  r0 = static_cast<int>(static_cast<unsigned>(c) * static_cast<unsigned>(n) / static_cast<unsigned>(g));
  r1 = static_cast<int>(static_cast<unsigned>(c + 1) * static_cast<unsigned>(n) / static_cast<unsigned>(g));
}

__device__ __forceinline__ void consumer_sync() { named_barrier_sync(1, kConsumers); }

// Consumer barrier that also tells every consumer whether this CTA has stopped; a CTA that stops sets the
// grid's abort word (sync[2]), so that the other CTAs leave their next barrier at once.
__device__ __forceinline__ bool consumers_stop(Ring& r, unsigned* sync) {
  const bool stop = named_barrier_or(1, kConsumers, r.abort != 0);
  if (stop && threadIdx.x == 0) atomicExch(sync + 2, 1u);
  return stop;
}

__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;"
      ::"r"(smem_addr(dst)), "l"(src), "r"(bytes), "r"(smem_addr(bar)), "l"(policy)
      : "memory");
}

__device__ __forceinline__ void unpack8(const uint4 v, float (&f)[8]) {
  f[0] = bf16lo(v.x); f[1] = bf16hi(v.x); f[2] = bf16lo(v.y); f[3] = bf16hi(v.y);
  f[4] = bf16lo(v.z); f[5] = bf16hi(v.z); f[6] = bf16lo(v.w); f[7] = bf16hi(v.w);
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  const __nv_bfloat162 p = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&p);
}

__device__ __forceinline__ uint4 pack8(const float (&o)[8]) {
  return make_uint4(pack_bf16x2(o[0], o[1]), pack_bf16x2(o[2], o[3]), pack_bf16x2(o[4], o[5]), pack_bf16x2(o[6], o[7]));
}

// 16 bytes through L2 (data written by other CTAs of the same launch).
__device__ __forceinline__ uint4 ldcg16(const void* p) { return __ldcg(reinterpret_cast<const uint4*>(p)); }

// 1 / sqrt(sum_sq / n + eps), each operation correctly rounded (decode.cu's RMSNorm).
__device__ __forceinline__ float inv_rms(float sum_sq, int n, float eps) {
  return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(sum_sq, static_cast<float>(n)), eps)));
}

// Sum over the 256 consumer threads in a fixed order (warp butterfly, then the warps in order).
__device__ __forceinline__ float consumer_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(kFull, v, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  consumer_sync();
  float t = 0.0f;
#pragma unroll
  for (int w = 0; w < kConsumerWarps; ++w) t += red[w];
  return t;
}

// Waits until ring chunk j has landed; nullptr when the CTA has stopped.
// An mbarrier wait names a phase by its parity only: waiting for use u of a slot returns at once while the
// slot is still in use u - 1 (use u - 2 has the same parity and has completed), which happens when a warp
// asks for chunk j before chunk j - kSlots has landed. So a warp first waits (bounded) until the producer
// has issued chunk j into the slot, which it does only after chunk j - kSlots was released, i.e. had
// landed; from then on the slot is in use u or later, and the parity wait is exact.
__device__ __forceinline__ const uint8_t* acquire(Ring& r, uint32_t j) {
  const uint32_t s = j % kSlots;
  volatile int* issued = r.issued;
  if (issued[s] < static_cast<int>(j)) {
    const unsigned long long t0 = globaltimer();
    for (uint32_t it = 1; issued[s] < static_cast<int>(j); ++it) {
      if ((it & 31u) == 0) {
        if (*reinterpret_cast<volatile int*>(&r.abort)) return nullptr;
        if (globaltimer() - t0 > kWaitLimitNs) {
          r.abort = 1;
          atomicOr(&g_bp_device_errors, BP_DEVERR_TIMEOUT);
          return nullptr;
        }
      }
    }
  }
  if (!mbar_wait(&r.full[s], (j / kSlots) & 1u, &r.abort)) return nullptr;
  return r.slot[s];
}

// The last of the `readers` warps done with ring chunk j gives its slot back to the producer.
__device__ __forceinline__ void release(Ring& r, uint32_t j, int readers) {
  __syncwarp();
  if ((threadIdx.x & 31) == 0) {
    const uint32_t s = j % kSlots;
    if (atomicAdd(&r.readers[s], 1) == readers - 1) {
      r.readers[s] = 0;
      mbar_arrive(&r.empty[s]);
    }
  }
}

// Grid barrier number `epoch` + 1 (consumers only): every CTA adds one to the arrival counter sync[0]
// (release: the CTA's global writes, ordered before it by the CTA barrier, become visible first) and waits
// (acquire) until the counter reaches (epoch + 1) * gridDim.x. The counter only grows during a launch (the
// host zeroes sync[0..3] before each launch). False when the step is aborted.
// ordered = false: the same without the release and acquire, a wake-up signal only, for hand-offs whose
// data carries its own readiness (glob_step.cu's tagged words): the release fence waited for the SM's bulk
// copies in flight, 1.2-1.7 us (measured with per-CTA stamps).
__device__ __forceinline__ bool grid_sync(Ring& r, unsigned* sync, unsigned& epoch, bool ordered = true) {
  consumer_sync();
  if (threadIdx.x == 0) {
    bool ok = true;
    const unsigned target = (epoch + 1) * gridDim.x;
    if (ordered)
      asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(sync) : "memory");
    else
      asm volatile("red.relaxed.gpu.global.add.u32 [%0], 1;" ::"l"(sync) : "memory");
    const unsigned long long t0 = globaltimer();
    for (uint32_t it = 0;; ++it) {
      unsigned v;
      if (ordered)
        asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(sync) : "memory");
      else
        asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(sync) : "memory");
      if (v >= target) break;
      if ((it & 63u) == 63u) {
        if (*reinterpret_cast<volatile unsigned*>(sync + 2) != 0u) {
          ok = false;
          break;
        }
        if (globaltimer() - t0 > kWaitLimitNs) {
          atomicExch(sync + 2, 1u);
          atomicOr(&g_bp_device_errors, BP_DEVERR_TIMEOUT);
          ok = false;
          break;
        }
      }
    }
    epoch += 1;
    r.bad = ok ? 0 : 1;
    if (!ok) r.abort = 1;
  }
  consumer_sync();
  return r.bad == 0;
}

// The producer: chunk k of `src` (src.chunk(k, bytes) -> global address) into the ring, k = 0 .. total-1;
// then waits for every copy in flight. No L2 prefetch ahead of the copies: with one prefetch per chunk the
// producer issued a chunk every 0.54 us instead of 0.32 (per-CTA stamps), which bounded the global step
// (682 against 621 us). Measured and not kept either: copying two contiguous chunks into neighbouring
// slots as one 32 KB operation (634 us), and requesting up to 12-48 chunks into L2 while the ring is full
// (614-640 us, against 575).
// Producer warp w of P (lane 0) issues the chunks k = w, w + P, ..., into slots k % kSlots (each warp its
// own slots, kSlots being a multiple of P). Two warps halve one issuing thread's latency per chunk: the
// local steps, whose phases are short, gained 52.3 -> 46.7 us; the global step lost (575 -> 627 us: its
// streams already keep HBM busy, and faster issue only adds to the queues its phase inputs wait in).
template <int P, typename Src>
__device__ void produce(Ring& r, const Src& src, int total, int w) {
  static_assert(kSlots % P == 0, "each producer warp owns whole slots");
  const uint64_t pol = l2_evict_first_policy();
  int k = w;
  for (; k < total; k += P) {
    const uint32_t s = k % kSlots, use = k / kSlots;
    uint32_t bytes;
    const void* p = src.chunk(k, bytes);  // before the wait: the copy leaves as soon as the slot is free
    if (use > 0 && !mbar_wait(&r.empty[s], (use - 1) & 1u, &r.abort)) break;
    mbar_arrive_expect_tx(&r.full[s], bytes);
    bulk_load(r.slot[s], p, bytes, &r.full[s], pol);
    *reinterpret_cast<volatile int*>(&r.issued[s]) = k;  // after the copy is on its way (see acquire)
  }
  int never = 0;  // every copy this warp issued (chunks w (mod P) below k) must land before exit
  for (int j = k - kSlots > w ? k - kSlots : w; j < k; j += P)
    mbar_wait(&r.full[j % kSlots], static_cast<uint32_t>(j / kSlots) & 1u, &never);
}

// ---- tagged hand-offs (the persistent steps) --------------------------------------------------------
// The outputs of the matrix-vector phases (y, o, a, dn) go to global memory as 32-bit words, the bf16 value
// in the low half and a 16-bit tag naming the write (launch number and hand-off) in the high half, each
// written by one relaxed store. The grid barrier between the phases is then only a wake-up signal (no
// release fence: it waited 1.2-1.7 us for the SM's bulk copies in flight, measured with per-CTA stamps), and
// a reader takes a word once it carries the expected tag, polling again in the rare case that the signal
// overtook the data. (Polling the words alone, without the signal, was slower: 256 threads per SM spinning on
// L2 loads delayed everything else.) Two writes to one word are at most a few hand-offs or one launch
// apart, so their tags always differ, and a zero-filled workspace never holds a valid tag.
__device__ __forceinline__ uint32_t hand_tag(unsigned seq, int t) { return 1u + (seq * 128u + t) % 65535u; }

__device__ __forceinline__ void st_tagged(uint32_t* p, float v, uint32_t tag) {
  const uint32_t w = (tag << 16) | static_cast<uint32_t>(__bfloat16_as_ushort(__float2bfloat16_rn(v)));
  asm volatile("st.relaxed.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(w) : "memory");
}

__device__ __forceinline__ uint4 ld_relaxed16(const uint32_t* p) {
  uint4 r;
  asm volatile("ld.relaxed.gpu.global.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p)
               : "memory");
  return r;
}

__device__ __forceinline__ uint32_t ld_relaxed4(const uint32_t* p) {
  uint32_t r;
  asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(r) : "l"(p) : "memory");
  return r;
}

// A failed tag wait: stop the grid (abort word; the device error flag when the wait timed out).
__device__ __forceinline__ bool tag_wait_gives_up(unsigned* sync, unsigned long long t0) {
  if (*reinterpret_cast<volatile unsigned*>(sync + 2) != 0u) return true;
  if (globaltimer() - t0 > kWaitLimitNs) {
    atomicExch(sync + 2, 1u);
    atomicOr(&g_bp_device_errors, BP_DEVERR_TIMEOUT);
    return true;
  }
  return false;
}

// The 8 tagged words at p (16-byte aligned), loaded already as u, v (so that a thread's loads are all in
// flight at once), once all carry `tag`, as floats (loading them again while one is stale); false when the
// step stops.
__device__ inline bool take_tagged8(uint4 u, uint4 v, const uint32_t* p, uint32_t tag, float (&f)[8], unsigned* sync) {
  auto ready = [&]() {
    return ((u.x >> 16) == tag) & ((u.y >> 16) == tag) & ((u.z >> 16) == tag) & ((u.w >> 16) == tag) &
           ((v.x >> 16) == tag) & ((v.y >> 16) == tag) & ((v.z >> 16) == tag) & ((v.w >> 16) == tag);
  };
  bool ok = true;
  if (!ready()) {
    const unsigned long long t0 = globaltimer();
    for (uint32_t it = 1;; ++it) {
      u = ld_relaxed16(p);
      v = ld_relaxed16(p + 4);
      if (ready()) break;
      if ((it & 31u) == 0 && tag_wait_gives_up(sync, t0)) {
        ok = false;
        break;
      }
    }
  }
  f[0] = __uint_as_float(u.x << 16); f[1] = __uint_as_float(u.y << 16);
  f[2] = __uint_as_float(u.z << 16); f[3] = __uint_as_float(u.w << 16);
  f[4] = __uint_as_float(v.x << 16); f[5] = __uint_as_float(v.y << 16);
  f[6] = __uint_as_float(v.z << 16); f[7] = __uint_as_float(v.w << 16);
  return ok;
}

__device__ __forceinline__ bool ld_tagged8(const uint32_t* p, uint32_t tag, float (&f)[8], unsigned* sync) {
  return take_tagged8(ld_relaxed16(p), ld_relaxed16(p + 4), p, tag, f, sync);
}

// One tagged word (loaded already as u) as a float, once it carries `tag`; false when the step stops.
__device__ inline bool take_tagged1(uint32_t u, const uint32_t* p, uint32_t tag, float& f, unsigned* sync) {
  bool ok = true;
  if ((u >> 16) != tag) {
    const unsigned long long t0 = globaltimer();
    for (uint32_t it = 1;; ++it) {
      u = ld_relaxed4(p);
      if ((u >> 16) == tag) break;
      if ((it & 31u) == 0 && tag_wait_gives_up(sync, t0)) {
        ok = false;
        break;
      }
    }
  }
  f = __uint_as_float(u << 16);
  return ok;
}

// Consumer barrier that stops the CTA when any consumer's wait failed (`bad`) or the ring stopped; a stop
// also stops this CTA's producer and tells the other CTAs (the grid's abort word).
__device__ __forceinline__ bool consumers_stop_if(Ring& r, unsigned* sync, bool bad) {
  const bool stop = named_barrier_or(1, kConsumers, bad || r.abort != 0);
  if (stop && threadIdx.x == 0) {
    r.abort = 1;
    atomicExch(sync + 2, 1u);
  }
  return stop;
}


// fp32 hand-off words (64 bits): the value's bits in the low half, the tag in the high half.
__device__ __forceinline__ void st_tagged_f32(uint64_t* p, float v, uint32_t tag) {
  const uint64_t w = (static_cast<uint64_t>(tag) << 32) | __float_as_uint(v);
  asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}

__device__ __forceinline__ uint64_t ld_relaxed8(const uint64_t* p) {
  uint64_t r;
  asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(r) : "l"(p) : "memory");
  return r;
}

// One fp32 hand-off word (loaded already as w) as a float, once it carries `tag`; false when the step stops.
__device__ inline bool take_tagged_f32(uint64_t w, const uint64_t* p, uint32_t tag, float& f, unsigned* sync) {
  bool ok = true;
  if (static_cast<uint32_t>(w >> 32) != tag) {
    const unsigned long long t0 = globaltimer();
    for (uint32_t it = 1;; ++it) {
      w = ld_relaxed8(p);
      if (static_cast<uint32_t>(w >> 32) == tag) break;
      if ((it & 31u) == 0 && tag_wait_gives_up(sync, t0)) {
        ok = false;
        break;
      }
    }
  }
  f = __uint_as_float(static_cast<uint32_t>(w));
  return ok;
}

// This lane's share of a 2048-vector in shared memory: x[lane * 8 + 256 i + j] -> xr[8 i + j].
__device__ __forceinline__ void load_lane_x(const __nv_bfloat16* vec, float (&xr)[64]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    float f[8];
    unpack8(*reinterpret_cast<const uint4*>(vec + lane * 8 + 256 * i), f);
#pragma unroll
    for (int j = 0; j < 8; ++j) xr[8 * i + j] = f[j];
  }
}

// The 4 rows of a K = 2048 chunk (bf16, in shared memory) . x at once (their loads and FMAs interleave),
// fp32, fixed order; every lane gets the 4 sums.
__device__ __forceinline__ void dot4x2048(const uint8_t* chunk, const float (&xr)[64], float (&out)[4]) {
  const int lane = threadIdx.x & 31;
  float acc[4][2];
#pragma unroll
  for (int r = 0; r < 4; ++r) acc[r][0] = acc[r][1] = 0.0f;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      float w[8];
      unpack8(*reinterpret_cast<const uint4*>(chunk + r * 4096 + (lane * 8 + 256 * i) * 2), w);
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[r][j & 1] = fmaf(w[j], xr[8 * i + j], acc[r][j & 1]);
    }
  }
#pragma unroll
  for (int r = 0; r < 4; ++r) out[r] = acc[r][0] + acc[r][1];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1)
#pragma unroll
    for (int r = 0; r < 4; ++r) out[r] += __shfl_xor_sync(kFull, out[r], o);
}

// v[lane] for lane < 4 (the lane's own row of a 4-row result).
__device__ __forceinline__ float lane_row(const float (&v)[4]) {
  const int lane = threadIdx.x & 31;
  float mine = v[0];
#pragma unroll
  for (int r = 1; r < 4; ++r) mine = lane == r ? v[r] : mine;
  return mine;
}

}  // namespace persist
}  // namespace bp
