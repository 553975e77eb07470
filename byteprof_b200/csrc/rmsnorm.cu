// Row-wise RMSNorm for the Bolmo-shaped local layers: y[r, :] = x[r, :] * rsqrt(mean(x[r, :]^2) + eps) * w.
//
// Reference: the pre-norms, per-head output norm and final norm of the local layers that byteprof's
// drafting engine runs over K + 1 positions (byteprof/optim/bolmo_draft.py:74-100).
//
// One warp per row; each lane sums the squares of its elements in a fixed order, then a fixed butterfly
// over the 32 lanes. The result of a row therefore does not depend on how many rows the launch holds,
// which the drafting check needs: verifying K drafts at once must give the same bits as K single steps.
// bf16 in and out, fp32 arithmetic, bf16 weight.
#include "bp_common.cuh"

namespace bp {
namespace {

constexpr int kWarpsPerCta = 8;

__global__ void __launch_bounds__(kWarpsPerCta * 32)
    rmsnorm_kernel(const __nv_bfloat16* __restrict__ x, long long ldx, const __nv_bfloat16* __restrict__ w,
                   __nv_bfloat16* __restrict__ y, long long ldy, int rows, int cols, float eps) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r = blockIdx.x * kWarpsPerCta + warp;
  if (r >= rows) return;
  const __nv_bfloat16* xr = x + static_cast<long long>(r) * ldx;
  __nv_bfloat16* yr = y + static_cast<long long>(r) * ldy;
  float ss = 0.0f;
  for (int c = lane * 8; c < cols; c += 32 * 8) {  // cols % 8 == 0, rows 16-byte aligned
    const uint4 v = *reinterpret_cast<const uint4*>(xr + c);
    const float f[8] = {bf16lo(v.x), bf16hi(v.x), bf16lo(v.y), bf16hi(v.y),
                        bf16lo(v.z), bf16hi(v.z), bf16lo(v.w), bf16hi(v.w)};
#pragma unroll
    for (int j = 0; j < 8; ++j) ss = fmaf(f[j], f[j], ss);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const float inv = rsqrtf(ss / static_cast<float>(cols) + eps);
  for (int c = lane * 8; c < cols; c += 32 * 8) {
    const uint4 v = *reinterpret_cast<const uint4*>(xr + c);
    const uint4 g = *reinterpret_cast<const uint4*>(w + c);
    const uint32_t xv[4] = {v.x, v.y, v.z, v.w}, gv[4] = {g.x, g.y, g.z, g.w};
    uint32_t o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float lo = bf16lo(xv[j]) * inv * bf16lo(gv[j]);
      const float hi = bf16hi(xv[j]) * inv * bf16hi(gv[j]);
      const __nv_bfloat162 p = __floats2bfloat162_rn(lo, hi);
      o[j] = *reinterpret_cast<const uint32_t*>(&p);
    }
    *reinterpret_cast<uint4*>(yr + c) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

}  // namespace
}  // namespace bp

extern "C" int bp_rmsnorm(const void* x, long long ldx, const void* w, void* y, long long ldy, int rows, int cols,
                          float eps, void* stream) {
  using namespace bp;
  clear_error();
  if (rows < 0 || cols < 0) return fail(BP_ERR_INVALID_ARGUMENT, "negative size (rows=%d cols=%d)", rows, cols);
  if (rows == 0 || cols == 0) return BP_OK;
  if (x == nullptr || w == nullptr || y == nullptr) return fail(BP_ERR_INVALID_ARGUMENT, "x, w or y is NULL");
  if (ldx < cols || ldy < cols) return fail(BP_ERR_INVALID_ARGUMENT, "row strides must be >= cols");
  if (cols % 8 != 0 || ldx % 8 != 0 || ldy % 8 != 0 || (reinterpret_cast<uintptr_t>(x) & 15u) ||
      (reinterpret_cast<uintptr_t>(w) & 15u) || (reinterpret_cast<uintptr_t>(y) & 15u))
    return fail(BP_ERR_MISALIGNED, "rmsnorm needs 16-byte aligned rows and cols, strides multiples of 8");
  int st = require_sm100();
  if (st != BP_OK) return st;
  const dim3 grid((rows + kWarpsPerCta - 1) / kWarpsPerCta);
  rmsnorm_kernel<<<grid, kWarpsPerCta * 32, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(x), ldx, static_cast<const __nv_bfloat16*>(w), static_cast<__nv_bfloat16*>(y),
      ldy, rows, cols, eps);
  return check_launch("rmsnorm");
}
