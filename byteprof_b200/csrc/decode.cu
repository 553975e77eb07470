// Glue kernels of the batch-1 byte decoder (a Bolmo-shaped model: mLSTM local layers around an
// OLMo-2 global model), each replacing a chain of small framework ops by one launch:
//   * bp_rmsnorm_ex   RMSNorm fused with the residual add that precedes it (pre-norm layers), the one
//                     that follows it (OLMo-2's norm-after blocks) or the mLSTM output gate; bp_rmsnorm
//                     is its plain mode;
//   * bp_swiglu       silu(gate) * up of a SwiGLU MLP;
//   * bp_gate_softcap cap * tanh((g + bias) / cap) of the mLSTM input / forget gate pre-activations;
//   * bp_decode_attention  one query position against a static KV cache: RMSNorm of q and k over the
//                     model width, rotary embedding, the cache write of k and v, and the attention
//                     split over a cluster of 8 CTAs per head, merged through distributed shared memory;
//   * bp_decode_finish the step's greedy argmax and boundary flag in one int64 pair.
// Reference: the per-byte pieces of byteprof's minimal Bolmo loop (byteprof/optim/bolmo.py:32-136,
// byteprof/optim/bolmo_loop.py:36-64), whose layers run these steps as separate framework ops.
//
// All kernels let the next kernel launch at once (programmatic dependent launch) and wait for the
// previous one before reading anything, so a following skinny GEMM streams its weights while these
// run. Activations (and the attention's KV cache) are bf16 or fp32 (`Act<T>`); weights are bf16.
// With bf16 activations the rounding points are those of the same steps written with bf16 torch
// tensors: every bf16 intermediate is rounded where a bf16 tensor would hold it, arithmetic in between
// is fp32. With fp32 activations nothing is rounded to bf16 (the decoder's exactness mode).
#include <math.h>

#include "bp_common.cuh"
#include "skinny_internal.h"
#include "sm100.cuh"

namespace bp {
namespace {

constexpr unsigned kFull = 0xffffffffu;

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  const __nv_bfloat162 p = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&p);
}

__device__ __forceinline__ void unpack8(const uint4 v, float (&f)[8]) {
  f[0] = bf16lo(v.x); f[1] = bf16hi(v.x); f[2] = bf16lo(v.y); f[3] = bf16hi(v.y);
  f[4] = bf16lo(v.z); f[5] = bf16hi(v.z); f[6] = bf16lo(v.w); f[7] = bf16hi(v.w);
}

// Activation element type: loads and stores of 8 consecutive values (16-byte aligned), single values,
// and the rounding a value of that type holds.
template <typename T>
struct Act;
template <>
struct Act<__nv_bfloat16> {
  static constexpr int kDtype = BP_DTYPE_BF16;
  __device__ static __forceinline__ void load8(const __nv_bfloat16* p, float (&f)[8]) { unpack8(ldg16(p), f); }
  __device__ static __forceinline__ void store8(__nv_bfloat16* p, const float (&f)[8]) {
    *reinterpret_cast<uint4*>(p) = make_uint4(pack_bf16x2(f[0], f[1]), pack_bf16x2(f[2], f[3]),
                                              pack_bf16x2(f[4], f[5]), pack_bf16x2(f[6], f[7]));
  }
  __device__ static __forceinline__ float load1(const __nv_bfloat16* p) { return __bfloat162float(*p); }
  __device__ static __forceinline__ void store1(__nv_bfloat16* p, float v) { *p = __float2bfloat16_rn(v); }
  __device__ static __forceinline__ float rnd(float v) { return round_bf16(v); }
};
template <>
struct Act<float> {
  static constexpr int kDtype = BP_DTYPE_F32;
  __device__ static __forceinline__ void load8(const float* p, float (&f)[8]) {
    const float4 a = __ldg(reinterpret_cast<const float4*>(p)), b = __ldg(reinterpret_cast<const float4*>(p) + 1);
    f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w; f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
  }
  __device__ static __forceinline__ void store8(float* p, const float (&f)[8]) {
    reinterpret_cast<float4*>(p)[0] = make_float4(f[0], f[1], f[2], f[3]);
    reinterpret_cast<float4*>(p)[1] = make_float4(f[4], f[5], f[6], f[7]);
  }
  __device__ static __forceinline__ float load1(const float* p) { return *p; }
  __device__ static __forceinline__ void store1(float* p, float v) { *p = v; }
  __device__ static __forceinline__ float rnd(float v) { return v; }
};

template <typename Kern, typename... Args>
cudaError_t launch_pdl(Kern kern, dim3 grid, dim3 block, cudaStream_t stream, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  cfg.numAttrs = 0;
  if (tc_pdl_enabled()) {
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.numAttrs = 1;
  }
  cfg.attrs = attr;
  return cudaLaunchKernelEx(&cfg, kern, args...);
}

// ---- RMSNorm with a fused add or gate ---------------------------------------------------------------
// One team of `team` threads (32 to 256) per row; a CTA holds 256 / team rows. Thread t of a team owns
// the 8-value chunks t, t + team, ... of its row and keeps up to kNormCache of them in registers, so a
// 2048-wide row is one 16-byte load per thread, all in flight at once. The sum of squares runs in a
// fixed order (each thread's chunks in order, a butterfly over the warp, the team's warps in order),
// so a row's result never depends on how many rows the launch holds. 1 / sqrt is two correctly
// rounded operations, reproducible on any IEEE machine.
constexpr int kNormThreads = 256;
constexpr int kNormCache = 4;

template <typename T>
struct NormArgs {
  const T* x;
  long long ldx;
  const __nv_bfloat16* w;
  int w_rows;
  const T* res;
  long long ldres;
  T* s_out;
  long long lds;
  T* y;
  long long ldy;
  int rows, cols;
  float eps;
  int team, iters;
  const long long* index;  // gather mode (PLAIN): row r of x is row index[r] of a table of index_rows rows
  long long index_rows;
};

// Row r = g * w_rows + j lives at g * ld + j * cols (w_rows = 1: the usual r * ld).
__device__ __forceinline__ long long row_off(int r, int w_rows, int cols, long long ld) {
  return static_cast<long long>(r / w_rows) * ld + static_cast<long long>(r % w_rows) * cols;
}

template <int MODE, typename T>
__device__ __forceinline__ void norm_in8(const T* xr, const T* rr, int c, float (&f)[8]) {
  Act<T>::load8(xr + c, f);
  if (MODE == BP_NORM_ADD_FIRST) {  // the normalised value is the sum as the activation type holds it
    float g[8];
    Act<T>::load8(rr + c, g);
#pragma unroll
    for (int j = 0; j < 8; ++j) f[j] = Act<T>::rnd(__fadd_rn(f[j], g[j]));
  }
}

// sigmoid evaluated in double precision and rounded once to fp32 (the correctly rounded value in all
// but rare cases), so that every implementation that does the same gets the same bits.
__device__ __forceinline__ float sigmoid_d(float v) { return static_cast<float>(1.0 / (1.0 + exp(-static_cast<double>(v)))); }

template <int MODE, typename T>
__device__ __forceinline__ void norm_out8(const float (&f)[8], float inv, const __nv_bfloat16* wr, const T* rr, T* sr,
                                          T* yr, int c) {
  float wv[8], o[8];
  unpack8(ldg16(wr + c), wv);
#pragma unroll
  for (int j = 0; j < 8; ++j) o[j] = __fmul_rn(__fmul_rn(f[j], inv), wv[j]);  // rounded to T by the store
  if (MODE == BP_NORM_ADD_AFTER || MODE == BP_NORM_GATE) {
    float e[8];
    Act<T>::load8(rr + c, e);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float nb = Act<T>::rnd(o[j]);
      o[j] = MODE == BP_NORM_ADD_AFTER ? __fadd_rn(e[j], nb) : __fmul_rn(Act<T>::rnd(sigmoid_d(e[j])), nb);
    }
  }
  if (sr != nullptr) Act<T>::store8(sr + c, f);
  Act<T>::store8(yr + c, o);
}

template <int MODE, bool kCached, typename T>
__global__ void __launch_bounds__(kNormThreads) norm_ex_kernel(NormArgs<T> a) {
  __shared__ float red[kNormThreads / 32];
  pdl_launch_dependents();
  pdl_wait_prior_grids();
  const int team = a.team, warps = team / 32;
  const int t = threadIdx.x % team, slot = threadIdx.x / team;
  const int r = blockIdx.x * (kNormThreads / team) + slot;
  const bool live = r < a.rows;
  const int rc = live ? r : a.rows - 1;  // rows past the end read the last row and store nothing
  const __nv_bfloat16* wr = a.w + static_cast<long long>(rc % a.w_rows) * a.cols;
  const T* xr = a.x + row_off(rc, a.w_rows, a.cols, a.ldx);
  bool poison = false;  // gather mode: an index outside the table gives a NaN row
  if (MODE == BP_NORM_PLAIN && a.index != nullptr) {
    const long long id = a.index[rc];
    poison = id < 0 || id >= a.index_rows;
    xr = a.x + (poison ? 0 : id) * a.ldx;
  }
  const T* rr = MODE == BP_NORM_PLAIN ? nullptr : a.res + row_off(rc, a.w_rows, a.cols, a.ldres);
  float f[kCached ? kNormCache : 1][8];
  float ss = 0.0f;
  auto load = [&](int c, float (&v)[8]) {
    norm_in8<MODE, T>(xr, rr, c, v);
    if (poison)
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = __int_as_float(0x7fc00000);
  };
  if (kCached) {
#pragma unroll
    for (int i = 0; i < kNormCache; ++i) {
      const int c = (t + i * team) * 8;
      if (i < a.iters && c < a.cols) {
        load(c, f[i]);
#pragma unroll
        for (int j = 0; j < 8; ++j) ss = fmaf(f[i][j], f[i][j], ss);
      }
    }
  } else {
    for (int c = t * 8; c < a.cols; c += team * 8) {
      load(c, f[0]);
#pragma unroll
      for (int j = 0; j < 8; ++j) ss = fmaf(f[0][j], f[0][j], ss);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(kFull, ss, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.0f;
  for (int w = 0; w < warps; ++w) tot += red[slot * warps + w];
  const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, static_cast<float>(a.cols)), a.eps)));
  if (!live) return;
  T* yr = a.y + row_off(r, a.w_rows, a.cols, a.ldy);
  // s_out: the sum (ADD_FIRST) or the gathered row (gather mode)
  T* sr = a.s_out != nullptr && (MODE == BP_NORM_ADD_FIRST || (MODE == BP_NORM_PLAIN && a.index != nullptr))
              ? a.s_out + row_off(r, a.w_rows, a.cols, a.lds)
              : nullptr;
  if (kCached) {
#pragma unroll
    for (int i = 0; i < kNormCache; ++i) {
      const int c = (t + i * team) * 8;
      if (i < a.iters && c < a.cols) norm_out8<MODE, T>(f[i], inv, wr, rr, sr, yr, c);
    }
  } else {
    for (int c = t * 8; c < a.cols; c += team * 8) {
      load(c, f[0]);
      norm_out8<MODE, T>(f[0], inv, wr, rr, sr, yr, c);
    }
  }
}

// ---- SwiGLU ---------------------------------------------------------------------------------------
// silu in double precision, rounded once to fp32, then to T; the product rounded to T by the store.
template <typename T>
__global__ void __launch_bounds__(256) swiglu_kernel(const T* __restrict__ gu, long long ldgu, T* __restrict__ out,
                                                     long long ldo, int ffn) {
  pdl_launch_dependents();
  pdl_wait_prior_grids();
  const int j = (blockIdx.x * blockDim.x + threadIdx.x) * 8;
  const int r = blockIdx.y;
  if (j >= ffn) return;
  const T* row = gu + static_cast<long long>(r) * ldgu;
  float g[8], u[8], o[8];
  Act<T>::load8(row + j, g);
  Act<T>::load8(row + ffn + j, u);
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    const float sl = Act<T>::rnd(static_cast<float>(g[q] / (1.0 + exp(-static_cast<double>(g[q])))));
    o[q] = __fmul_rn(sl, u[q]);
  }
  Act<T>::store8(out + static_cast<long long>(r) * ldo + j, o);
}

// ---- gate soft cap ----------------------------------------------------------------------------------
__global__ void __launch_bounds__(256) softcap_kernel(const float* g, long long ldg, const float* bias, float* out,
                                                      long long ldo, int rows, int n, float cap) {
  pdl_launch_dependents();
  pdl_wait_prior_grids();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= rows * n) return;
  const int r = i / n, c = i % n;
  const float t = __fadd_rn(g[static_cast<long long>(r) * ldg + c], bias != nullptr ? bias[c] : 0.0f);
  out[static_cast<long long>(r) * ldo + c] = __fmul_rn(cap, static_cast<float>(tanh(static_cast<double>(__fdiv_rn(t, cap)))));
}

// ---- single-position attention over a static KV cache -------------------------------------------------
// One thread-block cluster of 8 CTAs per head. CTA `rank` of head h takes positions rank * 128 .. +127 of
// every 1024-position round (warp w: 16 of them; lane: 4 of the 128 dims), keeps a running softmax (max,
// sum, unnormalised output) per warp, merges its 8 warps in shared memory and pushes the CTA's partial
// into slot `rank` of the leader CTA's shared memory (distributed shared memory); after one cluster
// barrier the leader merges the 8 slots in rank order (deterministic) and writes the head's output.
constexpr int kHd = 128;        // head dim
constexpr int kPerWarp = 16;    // positions per warp and round
constexpr int kAttnWarps = 8;
constexpr int kAttnThreads = kAttnWarps * 32;
constexpr int kCtaSpan = kAttnWarps * kPerWarp;   // 128 positions per CTA and round
constexpr int kAttnCluster = 8;                    // CTAs per head
constexpr int kRound = kAttnCluster * kCtaSpan;    // 1024 positions per round

template <typename T>
struct AttnArgs {
  const T* qkv;              // [3 * nh * kHd]: q | k | v of the current position
  const __nv_bfloat16* qw;   // q RMSNorm weight [nh * kHd]
  const __nv_bfloat16* kw;   // k RMSNorm weight [nh * kHd]
  const float* cos_t;        // [max_pos, kHd / 2]
  const float* sin_t;
  const long long* pos;      // device: the position of this query
  T* kc;                     // [max_pos, nh, kHd]
  T* vc;
  T* out;                    // [nh * kHd]
  int nh, max_pos;
  float eps, scale;
};

// Four consecutive cache values of one row as a lane holds them (8 bytes of bf16, 16 bytes of fp32).
template <typename T>
struct Row4;
template <>
struct Row4<__nv_bfloat16> {
  uint2 v;
  __device__ __forceinline__ void zero() { v = make_uint2(0u, 0u); }
  __device__ __forceinline__ void load(const __nv_bfloat16* p) { v = __ldg(reinterpret_cast<const uint2*>(p)); }
  __device__ __forceinline__ void get(float (&f)[4]) const {
    f[0] = bf16lo(v.x); f[1] = bf16hi(v.x); f[2] = bf16lo(v.y); f[3] = bf16hi(v.y);
  }
};
template <>
struct Row4<float> {
  float4 v;
  __device__ __forceinline__ void zero() { v = make_float4(0.f, 0.f, 0.f, 0.f); }
  __device__ __forceinline__ void load(const float* p) { v = __ldg(reinterpret_cast<const float4*>(p)); }
  __device__ __forceinline__ void get(float (&f)[4]) const { f[0] = v.x; f[1] = v.y; f[2] = v.z; f[3] = v.w; }
};


__device__ __forceinline__ float inv_rms(float sum_sq, int n, float eps) {
  return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(sum_sq, static_cast<float>(n)), eps)));
}

template <typename T>
__device__ __forceinline__ void load_rows(const AttnArgs<T>& a, long long base, long long p, int h, int lane,
                                          Row4<T> (&kk)[kPerWarp], Row4<T> (&vv)[kPerWarp]) {
#pragma unroll
  for (int j = 0; j < kPerWarp; ++j) {
    kk[j].zero();
    vv[j].zero();
    if (base + j < p) {  // rows below p were written by earlier launches; row p comes from this CTA
      const long long off = ((base + j) * a.nh + h) * kHd + lane * 4;
      kk[j].load(a.kc + off);
      vv[j].load(a.vc + off);
    }
  }
}

template <typename T>
__global__ void __cluster_dims__(kAttnCluster, 1, 1) __launch_bounds__(kAttnThreads)
    decode_attention_kernel(AttnArgs<T> a) {
  constexpr int kHalf = kHd / 2;
  __shared__ __align__(16) float qs[kHd];
  __shared__ __align__(16) float ks[kHd];  // position p's rotated k (bf16 values) and v, owner CTA only
  __shared__ __align__(16) float vs[kHd];
  __shared__ float red[2][kAttnWarps];
  __shared__ float wm[kAttnWarps], wl[kAttnWarps];
  __shared__ __align__(16) float wo[kAttnWarps][kHd];
  __shared__ float cm[kAttnCluster], cl[kAttnCluster];  // the leader's slots, one per CTA of the cluster
  __shared__ __align__(16) float co[kAttnCluster][kHd];
  pdl_launch_dependents();
  pdl_wait_prior_grids();
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int rank = static_cast<int>(cluster_ctarank()), h = blockIdx.y;
  const long long p = *a.pos;
  if (p < 0 || p >= a.max_pos) {  // the same p for the whole cluster: every CTA leaves here together
    if (rank == 0 && tid < kHd) Act<T>::store1(a.out + h * kHd + tid, __int_as_float(0x7fc00000));
    return;
  }
  const int rounds = static_cast<int>(p / kRound) + 1;
  const bool own = static_cast<int>((p % kRound) / kCtaSpan) == rank;  // this CTA's range holds p
  const int d = a.nh * kHd;
  const T* q = a.qkv;
  const T* k = a.qkv + d;
  const T* v = a.qkv + 2 * d;

  // Everything that depends only on p is requested first: round 0's cached rows of this warp, the
  // rotary factors, this head's q / k / v values and norm weights, the q and k vectors for the norms.
  Row4<T> kk[kPerWarp], vv[kPerWarp];
  load_rows(a, static_cast<long long>(rank) * kCtaSpan + warp * kPerWarp, p, h, lane, kk, vv);
  const int hi = h * kHd + (tid % kHalf);
  float cs = 0.0f, sn = 0.0f, qa = 0.0f, qb = 0.0f, qwa = 0.0f, qwb = 0.0f, ka = 0.0f, kb = 0.0f, kwa = 0.0f, kwb = 0.0f;
  float va = 0.0f, vb = 0.0f;
  if (tid < kHalf) {
    cs = a.cos_t[p * kHalf + tid];
    sn = a.sin_t[p * kHalf + tid];
    qa = Act<T>::load1(q + hi);
    qb = Act<T>::load1(q + hi + kHalf);
    qwa = __bfloat162float(a.qw[hi]);
    qwb = __bfloat162float(a.qw[hi + kHalf]);
    if (own) {
      ka = Act<T>::load1(k + hi);
      kb = Act<T>::load1(k + hi + kHalf);
      kwa = __bfloat162float(a.kw[hi]);
      kwb = __bfloat162float(a.kw[hi + kHalf]);
    }
  } else if (own && tid < kHd) {
    const int j = (tid - kHalf) * 2;
    va = Act<T>::load1(v + h * kHd + j);
    vb = Act<T>::load1(v + h * kHd + j + 1);
  }
  float sq = 0.0f, sk = 0.0f;
  for (int c = tid * 8; c < d; c += kAttnThreads * 8) {
    float fq[8], fk[8];
    Act<T>::load8(q + c, fq);
    Act<T>::load8(k + c, fk);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      sq = fmaf(fq[j], fq[j], sq);
      sk = fmaf(fk[j], fk[j], sk);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    sq += __shfl_xor_sync(kFull, sq, o);
    sk += __shfl_xor_sync(kFull, sk, o);
  }
  if (lane == 0) {
    red[0][warp] = sq;
    red[1][warp] = sk;
  }
  __syncthreads();
  float tq = 0.0f, tk = 0.0f;
#pragma unroll
  for (int w = 0; w < kAttnWarps; ++w) {
    tq += red[0][w];
    tk += red[1][w];
  }
  const float inv_q = inv_rms(tq, d, a.eps), inv_k = inv_rms(tk, d, a.eps);
  const long long slot = p * a.nh + h;  // cache row of (p, h)
  if (tid < kHalf) {
    const float q0 = Act<T>::rnd(__fmul_rn(__fmul_rn(qa, inv_q), qwa));
    const float q1 = Act<T>::rnd(__fmul_rn(__fmul_rn(qb, inv_q), qwb));
    qs[tid] = __fsub_rn(__fmul_rn(q0, cs), __fmul_rn(q1, sn));
    qs[tid + kHalf] = __fadd_rn(__fmul_rn(q1, cs), __fmul_rn(q0, sn));
    if (own) {
      const float k0 = Act<T>::rnd(__fmul_rn(__fmul_rn(ka, inv_k), kwa));
      const float k1 = Act<T>::rnd(__fmul_rn(__fmul_rn(kb, inv_k), kwb));
      const float r0 = Act<T>::rnd(__fsub_rn(__fmul_rn(k0, cs), __fmul_rn(k1, sn)));
      const float r1 = Act<T>::rnd(__fadd_rn(__fmul_rn(k1, cs), __fmul_rn(k0, sn)));
      Act<T>::store1(a.kc + slot * kHd + tid, r0);
      Act<T>::store1(a.kc + slot * kHd + tid + kHalf, r1);
      ks[tid] = r0;
      ks[tid + kHalf] = r1;
    }
  } else if (own && tid < kHd) {
    const int j = (tid - kHalf) * 2;
    Act<T>::store1(a.vc + slot * kHd + j, va);
    Act<T>::store1(a.vc + slot * kHd + j + 1, vb);
    vs[j] = va;
    vs[j + 1] = vb;
  }
  __syncthreads();  // qs (and ks, vs) visible to the whole CTA

  const float4 qv = *reinterpret_cast<const float4*>(&qs[lane * 4]);
  float mw = -INFINITY, lw = 0.0f, o4[4] = {0.0f, 0.0f, 0.0f, 0.0f};
  for (int r = 0; r < rounds; ++r) {
    const long long base = static_cast<long long>(r) * kRound + rank * kCtaSpan + warp * kPerWarp;
    if (r > 0) load_rows(a, base, p, h, lane, kk, vv);
    float sc[kPerWarp];
#pragma unroll
    for (int j = 0; j < kPerWarp; ++j) {
      float k4[4];
      if (base + j == p) {
        const float4 t = *reinterpret_cast<const float4*>(&ks[lane * 4]);
        k4[0] = t.x; k4[1] = t.y; k4[2] = t.z; k4[3] = t.w;
      } else {
        kk[j].get(k4);
      }
      float dot = __fmul_rn(qv.x, k4[0]);
      dot = fmaf(qv.y, k4[1], dot);
      dot = fmaf(qv.z, k4[2], dot);
      dot = fmaf(qv.w, k4[3], dot);
      sc[j] = dot;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
#pragma unroll
      for (int j = 0; j < kPerWarp; ++j) sc[j] += __shfl_xor_sync(kFull, sc[j], o);
    float mr = -INFINITY;
#pragma unroll
    for (int j = 0; j < kPerWarp; ++j) {
      sc[j] = base + j <= p ? __fmul_rn(sc[j], a.scale) : -INFINITY;
      mr = fmaxf(mr, sc[j]);
    }
    if (mr == -INFINITY) continue;  // no position of this round is at or below p (warp-uniform)
    const float m_new = fmaxf(mw, mr);
    if (mw != -INFINITY) {  // rescale what earlier rounds accumulated
      const float f = expf(__fsub_rn(mw, m_new));
      lw = __fmul_rn(lw, f);
#pragma unroll
      for (int c = 0; c < 4; ++c) o4[c] = __fmul_rn(o4[c], f);
    }
    mw = m_new;
    float e[kPerWarp];
#pragma unroll
    for (int j = 0; j < kPerWarp; ++j) e[j] = base + j <= p ? expf(__fsub_rn(sc[j], mw)) : 0.0f;
#pragma unroll
    for (int j = 0; j < kPerWarp; ++j) {
      if (base + j > p) continue;
      lw = __fadd_rn(lw, e[j]);
      float v4[4];
      if (base + j == p) {
        const float4 t = *reinterpret_cast<const float4*>(&vs[lane * 4]);
        v4[0] = t.x; v4[1] = t.y; v4[2] = t.z; v4[3] = t.w;
      } else {
        vv[j].get(v4);
      }
#pragma unroll
      for (int c = 0; c < 4; ++c) o4[c] = fmaf(e[j], v4[c], o4[c]);
    }
  }
  if (lane == 0) {
    wm[warp] = mw;
    wl[warp] = lw;
  }
  *reinterpret_cast<float4*>(&wo[warp][lane * 4]) = make_float4(o4[0], o4[1], o4[2], o4[3]);
  __syncthreads();
  // This CTA's partial (max, sum, output), pushed into slot `rank` of the leader CTA.
  if (tid < kHd) {
    float mc = -INFINITY;
#pragma unroll
    for (int w = 0; w < kAttnWarps; ++w) mc = fmaxf(mc, wm[w]);
    float lc = 0.0f, oc = 0.0f;
    if (mc != -INFINITY) {
#pragma unroll
      for (int w = 0; w < kAttnWarps; ++w) {
        const float f = wm[w] == -INFINITY ? 0.0f : expf(__fsub_rn(wm[w], mc));
        lc = fmaf(wl[w], f, lc);
        oc = fmaf(wo[w][tid], f, oc);
      }
    }
    const uint32_t dst_o = mapa_shared(smem_addr(&co[rank][tid]), 0);
    asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(dst_o), "f"(oc) : "memory");
    if (tid == 0) {
      asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(mapa_shared(smem_addr(&cm[rank]), 0)), "f"(mc) : "memory");
      asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(mapa_shared(smem_addr(&cl[rank]), 0)), "f"(lc) : "memory");
    }
  }
  cluster_sync_unaligned();  // every CTA's slot written (release) and visible to the leader (acquire)
  if (rank != 0 || tid >= kHd) return;
  float mg = -INFINITY;  // finite: rank 0's first position is 0 <= p
#pragma unroll
  for (int c = 0; c < kAttnCluster; ++c) mg = fmaxf(mg, cm[c]);
  float lg = 0.0f, og = 0.0f;
#pragma unroll
  for (int c = 0; c < kAttnCluster; ++c) {
    const float f = cm[c] == -INFINITY ? 0.0f : expf(__fsub_rn(cm[c], mg));
    lg = fmaf(cl[c], f, lg);
    og = fmaf(co[c][tid], f, og);
  }
  Act<T>::store1(a.out + h * kHd + tid, __fdiv_rn(og, lg));
}

// ---- argmax + boundary flag --------------------------------------------------------------------------
constexpr int kFinishThreads = 512;

// torch.argmax order: NaN is the largest value; ties go to the lowest index.
__device__ __forceinline__ bool better(float a, int ia, float b, int ib) {
  const bool na = isnan(a), nb = isnan(b);
  if (na || nb) return na && (!nb || ia < ib);
  return a > b || (a == b && ia < ib);
}

__global__ void __launch_bounds__(kFinishThreads) decode_finish_kernel(const float* logits, int n,
                                                                       const float* boundary_logit,
                                                                       long long* out) {
  __shared__ float bv[kFinishThreads / 32];
  __shared__ int bi[kFinishThreads / 32];
  pdl_launch_dependents();
  pdl_wait_prior_grids();
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  float best = -INFINITY;
  int idx = 0x7fffffff;
  for (int i = tid; i < n; i += kFinishThreads) {
    const float v = logits[i];
    if (better(v, i, best, idx)) {
      best = v;
      idx = i;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(kFull, best, o);
    const int oi = __shfl_xor_sync(kFull, idx, o);
    if (better(ov, oi, best, idx)) {
      best = ov;
      idx = oi;
    }
  }
  if (lane == 0) {
    bv[warp] = best;
    bi[warp] = idx;
  }
  __syncthreads();
  if (tid == 0) {
    for (int w = 1; w < kFinishThreads / 32; ++w)
      if (better(bv[w], bi[w], best, idx)) {
        best = bv[w];
        idx = bi[w];
      }
    out[0] = idx;
    out[1] = boundary_logit != nullptr && sigmoid_d(*boundary_logit) >= 0.5f ? 1 : 0;
  }
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

}  // namespace bp

namespace bp {
namespace {

template <int MODE, typename T>
cudaError_t launch_norm(NormArgs<T> a, cudaStream_t s) {
  int team = 32;  // threads per row: the power of two (32 to 256) covering cols / 8 chunks
  while (team < kNormThreads && team * 8 < a.cols) team *= 2;
  a.team = team;
  a.iters = (a.cols + team * 8 - 1) / (team * 8);
  const dim3 grid((a.rows + kNormThreads / team - 1) / (kNormThreads / team)), block(kNormThreads);
  return a.iters <= kNormCache ? launch_pdl(norm_ex_kernel<MODE, true, T>, grid, block, s, a)
                               : launch_pdl(norm_ex_kernel<MODE, false, T>, grid, block, s, a);
}

template <typename T>
cudaError_t launch_norm_mode(const void* x, long long ldx, const void* w, int w_rows, const void* res, long long ldres,
                             void* s_out, long long lds, void* y, long long ldy, int rows, int cols, float eps, int mode,
                             cudaStream_t s) {
  NormArgs<T> a{static_cast<const T*>(x), ldx, static_cast<const __nv_bfloat16*>(w), w_rows, static_cast<const T*>(res),
                ldres, static_cast<T*>(s_out), lds, static_cast<T*>(y), ldy, rows, cols, eps, 0, 0, nullptr, 0};
  switch (mode) {
    case BP_NORM_PLAIN: return launch_norm<BP_NORM_PLAIN, T>(a, s);
    case BP_NORM_ADD_FIRST: return launch_norm<BP_NORM_ADD_FIRST, T>(a, s);
    case BP_NORM_ADD_AFTER: return launch_norm<BP_NORM_ADD_AFTER, T>(a, s);
    default: return launch_norm<BP_NORM_GATE, T>(a, s);
  }
}

int check_act_dtype(int dtype) {
  if (dtype != BP_DTYPE_BF16 && dtype != BP_DTYPE_F32)
    return fail(BP_ERR_INVALID_ARGUMENT, "activation dtype %d is not bf16 or fp32", dtype);
  return BP_OK;
}

}  // namespace
}  // namespace bp

extern "C" int bp_rmsnorm_ex(const void* x, long long ldx, const void* w, int w_rows, const void* res, long long ldres,
                             void* s_out, long long lds, void* y, long long ldy, int rows, int cols, float eps, int mode,
                             int dtype, void* stream) {
  using namespace bp;
  clear_error();
  if (check_act_dtype(dtype) != BP_OK) return BP_ERR_INVALID_ARGUMENT;
  if (rows < 0 || cols < 0 || w_rows < 1)
    return fail(BP_ERR_INVALID_ARGUMENT, "bad size (rows=%d cols=%d w_rows=%d)", rows, cols, w_rows);
  if (mode < BP_NORM_PLAIN || mode > BP_NORM_GATE) return fail(BP_ERR_INVALID_ARGUMENT, "unknown norm mode %d", mode);
  if (rows == 0 || cols == 0) return BP_OK;
  if (x == nullptr || w == nullptr || y == nullptr || (mode != BP_NORM_PLAIN && res == nullptr))
    return fail(BP_ERR_INVALID_ARGUMENT, "x, w, y (or res for this mode) is NULL");
  if (s_out != nullptr && mode != BP_NORM_ADD_FIRST)
    return fail(BP_ERR_INVALID_ARGUMENT, "s_out is written by mode ADD_FIRST only");
  const long long span = static_cast<long long>(w_rows) * cols;  // a group of rows must fit its stride
  if (ldx < span || ldy < span || (mode != BP_NORM_PLAIN && ldres != 0 && ldres < span) ||
      (s_out != nullptr && lds < span))
    return fail(BP_ERR_INVALID_ARGUMENT, "row strides must cover a group of w_rows rows (ldres may be 0: broadcast)");
  if (cols % 8 != 0 || ldx % 8 != 0 || ldy % 8 != 0 || ldres % 8 != 0 || lds % 8 != 0 || !aligned16(x) ||
      !aligned16(w) || !aligned16(y) || (res != nullptr && !aligned16(res)) || (s_out != nullptr && !aligned16(s_out)))
    return fail(BP_ERR_MISALIGNED, "rmsnorm_ex needs 16-byte aligned rows, cols and strides multiples of 8");
  int st = require_sm100();
  if (st != BP_OK) return st;
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  const cudaError_t e =
      dtype == BP_DTYPE_BF16
          ? launch_norm_mode<__nv_bfloat16>(x, ldx, w, w_rows, res, ldres, s_out, lds, y, ldy, rows, cols, eps, mode, s)
          : launch_norm_mode<float>(x, ldx, w, w_rows, res, ldres, s_out, lds, y, ldy, rows, cols, eps, mode, s);
  if (e != cudaSuccess) return fail(BP_ERR_CUDA, "rmsnorm_ex launch: %s", cudaGetErrorString(e));
  return check_launch("rmsnorm_ex");
}

// Embedding lookup fused with the first norm of the byte encoder: h_out[r] = table[index[r]] and
// y[r] = rmsnorm(h_out[r]) * w, both bf16 (one launch instead of a gather kernel and a norm; the gather
// takes part in the PDL chain).
extern "C" int bp_embed_rmsnorm(const void* table, long long ld_table, long long table_rows, const int64_t* index,
                                const void* w, void* h_out, long long ldh, void* y, long long ldy, int rows, int cols,
                                float eps, void* stream) {
  using namespace bp;
  clear_error();
  if (rows < 0 || cols < 0 || table_rows < 0)
    return fail(BP_ERR_INVALID_ARGUMENT, "bad size (rows=%d cols=%d table_rows=%lld)", rows, cols, table_rows);
  if (rows == 0 || cols == 0) return BP_OK;
  if (table == nullptr || index == nullptr || w == nullptr || y == nullptr)
    return fail(BP_ERR_INVALID_ARGUMENT, "table, index, w or y is NULL");
  if (ld_table < cols || ldy < cols || (h_out != nullptr && ldh < cols))
    return fail(BP_ERR_INVALID_ARGUMENT, "row strides must be >= cols");
  if (cols % 8 != 0 || ld_table % 8 != 0 || ldy % 8 != 0 || ldh % 8 != 0 || !aligned16(table) || !aligned16(w) ||
      !aligned16(y) || (h_out != nullptr && !aligned16(h_out)) || (reinterpret_cast<uintptr_t>(index) & 7u) != 0)
    return fail(BP_ERR_MISALIGNED, "embed_rmsnorm needs 16-byte aligned rows, cols and strides multiples of 8");
  int st = require_sm100();
  if (st != BP_OK) return st;
  NormArgs<__nv_bfloat16> a{static_cast<const __nv_bfloat16*>(table), ld_table, static_cast<const __nv_bfloat16*>(w), 1,
                            nullptr, 0, static_cast<__nv_bfloat16*>(h_out), ldh, static_cast<__nv_bfloat16*>(y), ldy,
                            rows, cols, eps, 0, 0, reinterpret_cast<const long long*>(index), table_rows};
  const cudaError_t e = launch_norm<BP_NORM_PLAIN, __nv_bfloat16>(a, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return fail(BP_ERR_CUDA, "embed_rmsnorm launch: %s", cudaGetErrorString(e));
  return check_launch("embed_rmsnorm");
}

extern "C" int bp_rmsnorm(const void* x, long long ldx, const void* w, void* y, long long ldy, int rows, int cols,
                          float eps, void* stream) {
  return bp_rmsnorm_ex(x, ldx, w, 1, nullptr, 0, nullptr, 0, y, ldy, rows, cols, eps, BP_NORM_PLAIN, BP_DTYPE_BF16,
                       stream);
}

extern "C" int bp_swiglu(const void* gu, long long ldgu, void* out, long long ldo, int rows, int ffn, int dtype,
                         void* stream) {
  using namespace bp;
  clear_error();
  if (check_act_dtype(dtype) != BP_OK) return BP_ERR_INVALID_ARGUMENT;
  if (rows < 0 || ffn < 0) return fail(BP_ERR_INVALID_ARGUMENT, "negative size (rows=%d ffn=%d)", rows, ffn);
  if (rows == 0 || ffn == 0) return BP_OK;
  if (gu == nullptr || out == nullptr) return fail(BP_ERR_INVALID_ARGUMENT, "gu or out is NULL");
  if (ldgu < 2LL * ffn || ldo < ffn) return fail(BP_ERR_INVALID_ARGUMENT, "ldgu must be >= 2 * ffn and ldo >= ffn");
  if (ffn % 8 != 0 || ldgu % 8 != 0 || ldo % 8 != 0 || !aligned16(gu) || !aligned16(out))
    return fail(BP_ERR_MISALIGNED, "swiglu needs 16-byte aligned rows, ffn and strides multiples of 8");
  if (rows > 65535) return fail(BP_ERR_UNSUPPORTED, "swiglu takes at most 65535 rows per call");
  int st = require_sm100();
  if (st != BP_OK) return st;
  const dim3 grid((ffn / 8 + 255) / 256, rows);
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  const cudaError_t e =
      dtype == BP_DTYPE_BF16
          ? launch_pdl(swiglu_kernel<__nv_bfloat16>, grid, dim3(256), s, static_cast<const __nv_bfloat16*>(gu), ldgu,
                       static_cast<__nv_bfloat16*>(out), ldo, ffn)
          : launch_pdl(swiglu_kernel<float>, grid, dim3(256), s, static_cast<const float*>(gu), ldgu,
                       static_cast<float*>(out), ldo, ffn);
  if (e != cudaSuccess) return fail(BP_ERR_CUDA, "swiglu launch: %s", cudaGetErrorString(e));
  return check_launch("swiglu");
}

extern "C" int bp_gate_softcap(const float* g, long long ldg, const float* bias, float* out, long long ldo, int rows,
                               int n, float cap, void* stream) {
  using namespace bp;
  clear_error();
  if (rows < 0 || n < 0) return fail(BP_ERR_INVALID_ARGUMENT, "negative size (rows=%d n=%d)", rows, n);
  if (rows == 0 || n == 0) return BP_OK;
  if (g == nullptr || out == nullptr) return fail(BP_ERR_INVALID_ARGUMENT, "g or out is NULL");
  if (ldg < n || ldo < n) return fail(BP_ERR_INVALID_ARGUMENT, "row strides must be >= n");
  if (!(cap > 0.0f)) return fail(BP_ERR_INVALID_ARGUMENT, "cap must be positive");
  if (static_cast<long long>(rows) * n > (1LL << 30)) return fail(BP_ERR_UNSUPPORTED, "too many gate values");
  int st = require_sm100();
  if (st != BP_OK) return st;
  const int total = rows * n;
  const cudaError_t e = launch_pdl(softcap_kernel, dim3((total + 255) / 256), dim3(256),
                                   static_cast<cudaStream_t>(stream), g, ldg, bias, out, ldo, rows, n, cap);
  if (e != cudaSuccess) return fail(BP_ERR_CUDA, "gate_softcap launch: %s", cudaGetErrorString(e));
  return check_launch("gate_softcap");
}

namespace bp {
namespace {

template <typename T>
cudaError_t launch_attention(const void* qkv, const void* q_norm_w, const void* k_norm_w, const float* cos_t,
                             const float* sin_t, const int64_t* pos, void* k_cache, void* v_cache, void* out, int nh,
                             int max_pos, float eps, float scale, cudaStream_t s) {
  AttnArgs<T> a{static_cast<const T*>(qkv), static_cast<const __nv_bfloat16*>(q_norm_w),
                static_cast<const __nv_bfloat16*>(k_norm_w), cos_t, sin_t, reinterpret_cast<const long long*>(pos),
                static_cast<T*>(k_cache), static_cast<T*>(v_cache), static_cast<T*>(out), nh, max_pos, eps, scale};
  return launch_pdl(decode_attention_kernel<T>, dim3(kAttnCluster, nh), dim3(kAttnThreads), s, a);
}

}  // namespace
}  // namespace bp

extern "C" int bp_decode_attention(const void* qkv, const void* q_norm_w, const void* k_norm_w, const float* cos_t,
                                   const float* sin_t, const int64_t* pos, void* k_cache, void* v_cache, void* out,
                                   int nh, int head_dim, int max_pos, float eps, float scale, int dtype, void* stream) {
  using namespace bp;
  clear_error();
  if (check_act_dtype(dtype) != BP_OK) return BP_ERR_INVALID_ARGUMENT;
  if (head_dim != kHd) return fail(BP_ERR_UNSUPPORTED, "decode attention supports head_dim 128 (got %d)", head_dim);
  if (nh < 1 || nh > 65535 || max_pos < 1) return fail(BP_ERR_INVALID_ARGUMENT, "bad nh=%d or max_pos=%d", nh, max_pos);
  if (qkv == nullptr || q_norm_w == nullptr || k_norm_w == nullptr || cos_t == nullptr || sin_t == nullptr ||
      pos == nullptr || k_cache == nullptr || v_cache == nullptr || out == nullptr)
    return fail(BP_ERR_INVALID_ARGUMENT, "a pointer argument is NULL");
  if (!aligned16(qkv) || !aligned16(k_cache) || !aligned16(v_cache))
    return fail(BP_ERR_MISALIGNED, "qkv and the caches must be 16-byte aligned");
  int st = require_sm100();
  if (st != BP_OK) return st;
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  const cudaError_t e =
      dtype == BP_DTYPE_BF16
          ? launch_attention<__nv_bfloat16>(qkv, q_norm_w, k_norm_w, cos_t, sin_t, pos, k_cache, v_cache, out, nh,
                                            max_pos, eps, scale, s)
          : launch_attention<float>(qkv, q_norm_w, k_norm_w, cos_t, sin_t, pos, k_cache, v_cache, out, nh, max_pos,
                                    eps, scale, s);
  if (e != cudaSuccess) return fail(BP_ERR_CUDA, "decode_attention launch: %s", cudaGetErrorString(e));
  return check_launch("decode_attention");
}

extern "C" int bp_decode_finish(const float* logits, int n, const float* boundary_logit, int64_t* out, void* stream) {
  using namespace bp;
  clear_error();
  if (n < 1 || logits == nullptr || out == nullptr) return fail(BP_ERR_INVALID_ARGUMENT, "need n >= 1, logits and out");
  int st = require_sm100();
  if (st != BP_OK) return st;
  const cudaError_t e = launch_pdl(decode_finish_kernel, dim3(1), dim3(kFinishThreads), static_cast<cudaStream_t>(stream),
                                   logits, n, boundary_logit, reinterpret_cast<long long*>(out));
  if (e != cudaSuccess) return fail(BP_ERR_CUDA, "decode_finish launch: %s", cudaGetErrorString(e));
  return check_launch("decode_finish");
}
