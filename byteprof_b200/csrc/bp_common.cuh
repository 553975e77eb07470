// Shared plumbing of the byteprof B200 kernels: status/error reporting for the C ABI, dtype
// helpers and the few PTX wrappers the kernels use (streaming loads with an L2 evict-first policy,
// cp.async, bf16 packing).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdarg>
#include <cstdio>
#include <string>

#include "../../include/bp_kernels.h"

namespace bp {

// ---- error reporting (host) ---------------------------------------------------------------------
// One message per host thread; bp_last_error() returns it.
void set_error(const char* fmt, ...);
void clear_error();

// Returns `status` after recording a formatted message.
int fail(int status, const char* fmt, ...);

// Checks cudaGetLastError() after a launch; records the CUDA error string on failure.
int check_launch(const char* what);

// The current device must be sm_100 (B200 class); cached per device.
int require_sm100();

// Programmatic dependent launch: kernels launched with it start while the kernel before them in the
// stream still runs, and wait for it (pdl_wait_prior_grids) before touching anything it may write. On
// unless BP_DISABLE_PDL=1.
bool tc_pdl_enabled();

// Fills `attr` (room for two) with the PDL attribute (when enabled) and a cluster of `cluster_y` CTAs
// along y (when above 1), and points `cfg` at them.
inline void set_launch_attrs(cudaLaunchConfig_t& cfg, cudaLaunchAttribute* attr, int cluster_y = 1) {
  unsigned n = 0;
  if (tc_pdl_enabled()) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  if (cluster_y > 1) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = 1;
    attr[n].val.clusterDim.y = static_cast<unsigned>(cluster_y);
    attr[n].val.clusterDim.z = 1;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
}

// ---- device helpers -----------------------------------------------------------------------------
// Counterparts of set_launch_attrs' PDL attribute inside a kernel: let the next kernel's CTAs launch
// now (they wait on their side), and wait until every kernel before this one has finished and its
// writes are visible. Every kernel of a PDL chain waits before it reads or writes data another kernel
// touches, so one kernel's wait also covers all kernels before it.
__device__ __forceinline__ void pdl_wait_prior_grids() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

__device__ __forceinline__ float bf16lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

// Round-to-nearest-even fp32 -> bf16 -> fp32.
__device__ __forceinline__ float round_bf16(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }

// L2 policy: stream the weights through L2 with evict-first priority, so that they do not push out
// activations and other resident data (the reference loads its weight tiles with
// eviction_policy="evict_first", byteprof/optim/skinny.py:54,70).
__device__ __forceinline__ uint64_t l2_evict_first_policy() {
  uint64_t p;
  asm("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// L2 policy for data that should stay resident across kernels (the recurrent state of the decode loop,
// re-read at every byte while the weights stream through L2 evict-first).
__device__ __forceinline__ uint64_t l2_evict_last_policy() {
  uint64_t p;
  asm("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// 16-byte store with an L2 cache policy.
__device__ __forceinline__ void st_global16_hint(void* ptr, const float4& v, uint64_t policy) {
  asm volatile("st.global.L2::cache_hint.v4.f32 [%0], {%1, %2, %3, %4}, %5;" ::"l"(ptr), "f"(v.x), "f"(v.y), "f"(v.z),
               "f"(v.w), "l"(policy)
               : "memory");
}

// 16-byte read-only streaming load: not allocated in L1, evict-first in L2.
__device__ __forceinline__ uint4 ldg_stream16(const void* ptr, uint64_t policy) {
  uint4 r;
  asm("ld.global.nc.L1::no_allocate.L2::cache_hint.v4.u32 {%0, %1, %2, %3}, [%4], %5;"
      : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
      : "l"(ptr), "l"(policy));
  return r;
}

// 16-byte read-only load through L1 (small operands re-read by many warps: activations).
__device__ __forceinline__ uint4 ldg16(const void* ptr) {
  uint4 r;
  asm("ld.global.nc.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(ptr));
  return r;
}

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// Ampere-style asynchronous global -> shared copies (16 bytes), grouped with commit/wait.
__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(smem)), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async16_hint(void* smem, const void* gmem, uint64_t policy) {
  asm volatile("cp.async.cg.shared.global.L2::cache_hint [%0], [%1], 16, %2;" ::"r"(smem_addr(smem)), "l"(gmem),
               "l"(policy)
               : "memory");
}
__device__ __forceinline__ void cp_async4(void* smem, const void* gmem) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_addr(smem)), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

}  // namespace bp
