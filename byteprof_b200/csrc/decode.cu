// Glue kernels of the batch-1 byte decoder (a Bolmo-shaped model: mLSTM local layers around an
// OLMo-2 global model), each replacing a chain of small framework ops by one launch:
//   * bp_rmsnorm_ex   RMSNorm fused with the residual add that precedes it (pre-norm layers), the one
//                     that follows it (OLMo-2's norm-after blocks) or the mLSTM output gate;
//   * bp_swiglu       silu(gate) * up of a SwiGLU MLP;
//   * bp_gate_softcap cap * tanh((g + bias) / cap) of the mLSTM input / forget gate pre-activations;
//   * bp_decode_attention  one query position against a static KV cache: RMSNorm of q and k over the
//                     model width, rotary embedding, the cache write of k and v, and the attention
//                     split over 64-position chunks with a deterministic last-arriver combine;
//   * bp_decode_finish the step's greedy argmax and boundary flag in one int64 pair.
// Reference: the per-byte pieces of byteprof's minimal Bolmo loop (byteprof/optim/bolmo.py:32-136,
// byteprof/optim/bolmo_loop.py:36-64), whose layers run these steps as separate framework ops.
//
// All kernels let the next kernel launch at once (programmatic dependent launch) and wait for the
// previous one before reading anything, so a following skinny GEMM streams its weights while these
// run. Rounding points are those of the same steps written with bf16 torch tensors: every bf16
// intermediate is rounded where a bf16 tensor would hold it; arithmetic in between is fp32.
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

__device__ __forceinline__ float sigmoid_f(float v) { return 1.0f / (1.0f + expf(-v)); }

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
constexpr int kNormWarps = 8;

struct NormArgs {
  const __nv_bfloat16* x;
  long long ldx;
  const __nv_bfloat16* w;
  int w_rows;
  const __nv_bfloat16* res;
  long long ldres;
  __nv_bfloat16* s_out;
  long long lds;
  __nv_bfloat16* y;
  long long ldy;
  int rows, cols;
  float eps;
};

// Row r = g * w_rows + j lives at g * ld + j * cols (w_rows = 1: the usual r * ld).
__device__ __forceinline__ long long row_off(int r, int w_rows, int cols, long long ld) {
  return static_cast<long long>(r / w_rows) * ld + static_cast<long long>(r % w_rows) * cols;
}

template <int MODE>
__device__ __forceinline__ void norm_in8(const __nv_bfloat16* xr, const __nv_bfloat16* rr, int c, float (&f)[8]) {
  const uint4 v = ldg16(xr + c);
  f[0] = bf16lo(v.x); f[1] = bf16hi(v.x); f[2] = bf16lo(v.y); f[3] = bf16hi(v.y);
  f[4] = bf16lo(v.z); f[5] = bf16hi(v.z); f[6] = bf16lo(v.w); f[7] = bf16hi(v.w);
  if (MODE == BP_NORM_ADD_FIRST) {  // the normalised value is the bf16 sum
    const uint4 u = ldg16(rr + c);
    const float g[8] = {bf16lo(u.x), bf16hi(u.x), bf16lo(u.y), bf16hi(u.y),
                        bf16lo(u.z), bf16hi(u.z), bf16lo(u.w), bf16hi(u.w)};
#pragma unroll
    for (int j = 0; j < 8; ++j) f[j] = round_bf16(__fadd_rn(f[j], g[j]));
  }
}

template <int MODE>
__global__ void __launch_bounds__(kNormWarps * 32) norm_ex_kernel(NormArgs a) {
  pdl_launch_dependents();
  pdl_wait_prior_grids();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r = blockIdx.x * kNormWarps + warp;
  if (r >= a.rows) return;
  const __nv_bfloat16* wr = a.w + static_cast<long long>(r % a.w_rows) * a.cols;
  const __nv_bfloat16* xr = a.x + row_off(r, a.w_rows, a.cols, a.ldx);
  const __nv_bfloat16* rr = MODE == BP_NORM_PLAIN ? nullptr : a.res + row_off(r, a.w_rows, a.cols, a.ldres);
  __nv_bfloat16* yr = a.y + row_off(r, a.w_rows, a.cols, a.ldy);
  __nv_bfloat16* sr = (MODE == BP_NORM_ADD_FIRST && a.s_out != nullptr) ? a.s_out + row_off(r, a.w_rows, a.cols, a.lds)
                                                                        : nullptr;
  float ss = 0.0f;
  for (int c = lane * 8; c < a.cols; c += 32 * 8) {  // the same per-lane order as bp_rmsnorm
    float f[8];
    norm_in8<MODE>(xr, rr, c, f);
#pragma unroll
    for (int j = 0; j < 8; ++j) ss = fmaf(f[j], f[j], ss);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(kFull, ss, o);
  const float inv = rsqrtf(ss / static_cast<float>(a.cols) + a.eps);
  for (int c = lane * 8; c < a.cols; c += 32 * 8) {
    float f[8];
    norm_in8<MODE>(xr, rr, c, f);
    const uint4 g = ldg16(wr + c);
    const float wv[8] = {bf16lo(g.x), bf16hi(g.x), bf16lo(g.y), bf16hi(g.y),
                         bf16lo(g.z), bf16hi(g.z), bf16lo(g.w), bf16hi(g.w)};
    float o[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j] = __fmul_rn(__fmul_rn(f[j], inv), wv[j]);  // bf16(x * inv * w) below
    if (MODE == BP_NORM_ADD_AFTER || MODE == BP_NORM_GATE) {
      const uint4 u = ldg16(rr + c);
      const float e[8] = {bf16lo(u.x), bf16hi(u.x), bf16lo(u.y), bf16hi(u.y),
                          bf16lo(u.z), bf16hi(u.z), bf16lo(u.w), bf16hi(u.w)};
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float nb = round_bf16(o[j]);
        o[j] = MODE == BP_NORM_ADD_AFTER ? __fadd_rn(e[j], nb) : __fmul_rn(round_bf16(sigmoid_f(e[j])), nb);
      }
    }
    if (sr != nullptr)
      *reinterpret_cast<uint4*>(sr + c) = make_uint4(pack_bf16x2(f[0], f[1]), pack_bf16x2(f[2], f[3]),
                                                     pack_bf16x2(f[4], f[5]), pack_bf16x2(f[6], f[7]));
    *reinterpret_cast<uint4*>(yr + c) = make_uint4(pack_bf16x2(o[0], o[1]), pack_bf16x2(o[2], o[3]),
                                                   pack_bf16x2(o[4], o[5]), pack_bf16x2(o[6], o[7]));
  }
}

// ---- SwiGLU ---------------------------------------------------------------------------------------
__global__ void __launch_bounds__(256) swiglu_kernel(const __nv_bfloat16* __restrict__ gu, long long ldgu,
                                                     __nv_bfloat16* __restrict__ out, long long ldo, int ffn) {
  pdl_launch_dependents();
  pdl_wait_prior_grids();
  const int j = (blockIdx.x * blockDim.x + threadIdx.x) * 8;
  const int r = blockIdx.y;
  if (j >= ffn) return;
  const __nv_bfloat16* row = gu + static_cast<long long>(r) * ldgu;
  const uint4 g = ldg16(row + j), u = ldg16(row + ffn + j);
  const uint32_t gv[4] = {g.x, g.y, g.z, g.w}, uv[4] = {u.x, u.y, u.z, u.w};
  uint32_t o[4];
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const float g0 = bf16lo(gv[q]), g1 = bf16hi(gv[q]);
    const float s0 = round_bf16(g0 / (1.0f + expf(-g0))), s1 = round_bf16(g1 / (1.0f + expf(-g1)));
    o[q] = pack_bf16x2(__fmul_rn(s0, bf16lo(uv[q])), __fmul_rn(s1, bf16hi(uv[q])));
  }
  *reinterpret_cast<uint4*>(out + static_cast<long long>(r) * ldo + j) = make_uint4(o[0], o[1], o[2], o[3]);
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
  out[static_cast<long long>(r) * ldo + c] = __fmul_rn(cap, tanhf(__fdiv_rn(t, cap)));
}

// ---- single-position attention over a static KV cache -------------------------------------------------
constexpr int kHd = 128;        // head dim
constexpr int kChunk = 64;      // positions per CTA
constexpr int kPerWarp = 16;    // positions per warp
constexpr int kAttnThreads = 128;
static_assert(kChunk == kPerWarp * kAttnThreads / 32, "chunk = 4 warps x 16 positions");

struct AttnArgs {
  const __nv_bfloat16* qkv;  // [3 * nh * kHd]: q | k | v of the current position
  const __nv_bfloat16* qw;   // q RMSNorm weight [nh * kHd]
  const __nv_bfloat16* kw;   // k RMSNorm weight [nh * kHd]
  const float* cos_t;        // [max_pos, kHd / 2]
  const float* sin_t;
  const long long* pos;      // device: the position of this query
  __nv_bfloat16* kc;         // [max_pos, nh, kHd]
  __nv_bfloat16* vc;
  __nv_bfloat16* out;        // [nh * kHd]
  float* part;               // [nh][max_chunks][kHd + 2]: chunk max, sum, unnormalised output
  unsigned* counters;        // [nh], zero between launches
  int nh, max_pos, max_chunks;
  float eps, scale;
};

__device__ __forceinline__ float block_sum4(float v, float* red) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(kFull, v, o);
  if (lane == 0) red[warp] = v;
  __syncthreads();
  return ((red[0] + red[1]) + red[2]) + red[3];
}

__global__ void __launch_bounds__(kAttnThreads) decode_attention_kernel(AttnArgs a) {
  __shared__ __align__(16) float qs[kHd];
  __shared__ float red[2][4];
  __shared__ float wm[4], wl[4];
  __shared__ __align__(16) float wo[4][kHd];
  __shared__ int is_last;
  pdl_launch_dependents();
  pdl_wait_prior_grids();
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int chunk = blockIdx.x, h = blockIdx.y;
  const long long p = *a.pos;
  if (p < 0 || p >= a.max_pos) {  // host-side checks keep p in range; never index with a bad one
    if (chunk == 0) a.out[h * kHd + tid] = __float2bfloat16_rn(__int_as_float(0x7fc00000));
    return;
  }
  const int nchunks = static_cast<int>(p / kChunk) + 1;
  if (chunk >= nchunks) return;
  const bool own = chunk == nchunks - 1;  // this CTA's range holds position p
  const int d = a.nh * kHd;
  const __nv_bfloat16* q = a.qkv;
  const __nv_bfloat16* k = a.qkv + d;
  const __nv_bfloat16* v = a.qkv + 2 * d;

  float sq = 0.0f, sk = 0.0f;
  for (int c = tid * 8; c < d; c += kAttnThreads * 8) {
    const uint4 qv = ldg16(q + c), kv = ldg16(k + c);
    const uint32_t qa[4] = {qv.x, qv.y, qv.z, qv.w}, ka[4] = {kv.x, kv.y, kv.z, kv.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      sq = fmaf(bf16lo(qa[j]), bf16lo(qa[j]), sq);
      sq = fmaf(bf16hi(qa[j]), bf16hi(qa[j]), sq);
      sk = fmaf(bf16lo(ka[j]), bf16lo(ka[j]), sk);
      sk = fmaf(bf16hi(ka[j]), bf16hi(ka[j]), sk);
    }
  }
  const float tq = block_sum4(sq, red[0]);
  const float tk = block_sum4(sk, red[1]);
  const float inv_q = rsqrtf(tq / static_cast<float>(d) + a.eps);
  const float inv_k = rsqrtf(tk / static_cast<float>(d) + a.eps);
  const long long slot = p * a.nh + h;  // cache row of (p, h)
  if (tid < kHd / 2) {
    const int i0 = h * kHd + tid, i1 = i0 + kHd / 2;
    const float cs = a.cos_t[p * (kHd / 2) + tid], sn = a.sin_t[p * (kHd / 2) + tid];
    const float q0 = round_bf16(__fmul_rn(__fmul_rn(__bfloat162float(q[i0]), inv_q), __bfloat162float(a.qw[i0])));
    const float q1 = round_bf16(__fmul_rn(__fmul_rn(__bfloat162float(q[i1]), inv_q), __bfloat162float(a.qw[i1])));
    qs[tid] = __fsub_rn(__fmul_rn(q0, cs), __fmul_rn(q1, sn));
    qs[tid + kHd / 2] = __fadd_rn(__fmul_rn(q1, cs), __fmul_rn(q0, sn));
    if (own) {
      const float k0 = round_bf16(__fmul_rn(__fmul_rn(__bfloat162float(k[i0]), inv_k), __bfloat162float(a.kw[i0])));
      const float k1 = round_bf16(__fmul_rn(__fmul_rn(__bfloat162float(k[i1]), inv_k), __bfloat162float(a.kw[i1])));
      a.kc[slot * kHd + tid] = __float2bfloat16_rn(__fsub_rn(__fmul_rn(k0, cs), __fmul_rn(k1, sn)));
      a.kc[slot * kHd + tid + kHd / 2] = __float2bfloat16_rn(__fadd_rn(__fmul_rn(k1, cs), __fmul_rn(k0, sn)));
    }
  } else if (own) {
    const int j = (tid - kHd / 2) * 2;
    a.vc[slot * kHd + j] = v[h * kHd + j];
    a.vc[slot * kHd + j + 1] = v[h * kHd + j + 1];
  }
  __syncthreads();  // qs, and this CTA's cache writes, visible to the whole CTA

  // Scores: warp w takes positions base .. base + 15; lane holds dims 4 * lane .. 4 * lane + 3.
  // Plain loads: the cache row of p was written by this CTA in this launch.
  const long long base = static_cast<long long>(chunk) * kChunk + warp * kPerWarp;
  const float4 qv = *reinterpret_cast<const float4*>(&qs[lane * 4]);
  float sc[kPerWarp];
#pragma unroll
  for (int j = 0; j < kPerWarp; ++j) {
    float dot = 0.0f;
    if (base + j <= p) {
      const uint2 kk = *reinterpret_cast<const uint2*>(a.kc + ((base + j) * a.nh + h) * kHd + lane * 4);
      dot = __fmul_rn(qv.x, bf16lo(kk.x));
      dot = fmaf(qv.y, bf16hi(kk.x), dot);
      dot = fmaf(qv.z, bf16lo(kk.y), dot);
      dot = fmaf(qv.w, bf16hi(kk.y), dot);
    }
    sc[j] = dot;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1)
#pragma unroll
    for (int j = 0; j < kPerWarp; ++j) sc[j] += __shfl_xor_sync(kFull, sc[j], o);
  float mw = -INFINITY;
#pragma unroll
  for (int j = 0; j < kPerWarp; ++j) {
    sc[j] = base + j <= p ? sc[j] * a.scale : -INFINITY;
    mw = fmaxf(mw, sc[j]);
  }
  float lw = 0.0f, o4[4] = {0.0f, 0.0f, 0.0f, 0.0f};
  if (mw != -INFINITY) {
#pragma unroll
    for (int j = 0; j < kPerWarp; ++j) {
      if (base + j > p) continue;
      const float e = expf(sc[j] - mw);
      lw += e;
      const uint2 vv = *reinterpret_cast<const uint2*>(a.vc + ((base + j) * a.nh + h) * kHd + lane * 4);
      o4[0] = fmaf(e, bf16lo(vv.x), o4[0]);
      o4[1] = fmaf(e, bf16hi(vv.x), o4[1]);
      o4[2] = fmaf(e, bf16lo(vv.y), o4[2]);
      o4[3] = fmaf(e, bf16hi(vv.y), o4[3]);
    }
  }
  if (lane == 0) {
    wm[warp] = mw;
    wl[warp] = lw;
  }
  *reinterpret_cast<float4*>(&wo[warp][lane * 4]) = make_float4(o4[0], o4[1], o4[2], o4[3]);
  __syncthreads();
  // Chunk partial (warp 0's first position is chunk * 64 <= p, so the chunk max is finite).
  const float mc = fmaxf(fmaxf(wm[0], wm[1]), fmaxf(wm[2], wm[3]));
  float lc = 0.0f, oc = 0.0f;
#pragma unroll
  for (int w = 0; w < 4; ++w) {
    const float f = wm[w] == -INFINITY ? 0.0f : expf(wm[w] - mc);
    lc = fmaf(wl[w], f, lc);
    oc = fmaf(wo[w][tid], f, oc);
  }
  float* ph = a.part + static_cast<long long>(h) * a.max_chunks * (kHd + 2);
  float* pc = ph + static_cast<long long>(chunk) * (kHd + 2);
  pc[2 + tid] = oc;
  if (tid == 0) {
    pc[0] = mc;
    pc[1] = lc;
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) is_last = atomicAdd(&a.counters[h], 1u) == static_cast<unsigned>(nchunks - 1);
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  // The last CTA of head h combines all chunks in chunk order (deterministic).
  float mg = -INFINITY;
  for (int c = 0; c < nchunks; ++c) mg = fmaxf(mg, __ldcg(ph + static_cast<long long>(c) * (kHd + 2)));
  float lg = 0.0f, og = 0.0f;
  for (int c = 0; c < nchunks; ++c) {
    const float* pp = ph + static_cast<long long>(c) * (kHd + 2);
    const float f = expf(__ldcg(pp) - mg);
    lg = fmaf(__ldcg(pp + 1), f, lg);
    og = fmaf(__ldcg(pp + 2 + tid), f, og);
  }
  a.out[h * kHd + tid] = __float2bfloat16_rn(og / lg);
  if (tid == 0) a.counters[h] = 0u;
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
    out[1] = boundary_logit != nullptr && sigmoid_f(*boundary_logit) >= 0.5f ? 1 : 0;
  }
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

size_t decode_attention_workspace_bytes(int nh, int max_pos) {
  const size_t chunks = static_cast<size_t>((max_pos + kChunk - 1) / kChunk);
  const size_t part = static_cast<size_t>(nh) * chunks * (kHd + 2) * sizeof(float);
  return ((part + 255) / 256) * 256 + static_cast<size_t>(nh) * sizeof(unsigned);
}

}  // namespace bp

extern "C" int bp_rmsnorm_ex(const void* x, long long ldx, const void* w, int w_rows, const void* res, long long ldres, void* s_out, long long lds, void* y,
                             long long ldy, int rows, int cols, float eps, int mode, void* stream) {
  using namespace bp;
  clear_error();
  if (rows < 0 || cols < 0 || w_rows < 1) return fail(BP_ERR_INVALID_ARGUMENT, "bad size (rows=%d cols=%d w_rows=%d)", rows, cols, w_rows);
  if (mode < BP_NORM_PLAIN || mode > BP_NORM_GATE) return fail(BP_ERR_INVALID_ARGUMENT, "unknown norm mode %d", mode);
  if (rows == 0 || cols == 0) return BP_OK;
  if (x == nullptr || w == nullptr || y == nullptr || (mode != BP_NORM_PLAIN && res == nullptr))
    return fail(BP_ERR_INVALID_ARGUMENT, "x, w, y (or res for this mode) is NULL");
  if (s_out != nullptr && mode != BP_NORM_ADD_FIRST) return fail(BP_ERR_INVALID_ARGUMENT, "s_out is written by mode ADD_FIRST only");
  const long long span = static_cast<long long>(w_rows) * cols;  // a group of rows must fit its stride
  if (ldx < span || ldy < span || (mode != BP_NORM_PLAIN && ldres != 0 && ldres < span) ||
      (s_out != nullptr && lds < span))
    return fail(BP_ERR_INVALID_ARGUMENT, "row strides must cover a group of w_rows rows (ldres may be 0: broadcast)");
  if (cols % 8 != 0 || ldx % 8 != 0 || ldy % 8 != 0 || ldres % 8 != 0 || lds % 8 != 0 || !aligned16(x) ||
      !aligned16(w) || !aligned16(y) || (res != nullptr && !aligned16(res)) || (s_out != nullptr && !aligned16(s_out)))
    return fail(BP_ERR_MISALIGNED, "rmsnorm_ex needs 16-byte aligned rows, cols and strides multiples of 8");
  int st = require_sm100();
  if (st != BP_OK) return st;
  NormArgs a{static_cast<const __nv_bfloat16*>(x), ldx, static_cast<const __nv_bfloat16*>(w), w_rows, static_cast<const __nv_bfloat16*>(res), ldres,
             static_cast<__nv_bfloat16*>(s_out), lds, static_cast<__nv_bfloat16*>(y), ldy, rows, cols, eps};
  const dim3 grid((rows + kNormWarps - 1) / kNormWarps), block(kNormWarps * 32);
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e;
  switch (mode) {
    case BP_NORM_PLAIN: e = launch_pdl(norm_ex_kernel<BP_NORM_PLAIN>, grid, block, s, a); break;
    case BP_NORM_ADD_FIRST: e = launch_pdl(norm_ex_kernel<BP_NORM_ADD_FIRST>, grid, block, s, a); break;
    case BP_NORM_ADD_AFTER: e = launch_pdl(norm_ex_kernel<BP_NORM_ADD_AFTER>, grid, block, s, a); break;
    default: e = launch_pdl(norm_ex_kernel<BP_NORM_GATE>, grid, block, s, a); break;
  }
  if (e != cudaSuccess) return fail(BP_ERR_CUDA, "rmsnorm_ex launch: %s", cudaGetErrorString(e));
  return check_launch("rmsnorm_ex");
}

extern "C" int bp_swiglu(const void* gu, long long ldgu, void* out, long long ldo, int rows, int ffn, void* stream) {
  using namespace bp;
  clear_error();
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
  const cudaError_t e = launch_pdl(swiglu_kernel, grid, dim3(256), static_cast<cudaStream_t>(stream),
                                   static_cast<const __nv_bfloat16*>(gu), ldgu, static_cast<__nv_bfloat16*>(out), ldo, ffn);
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

extern "C" size_t bp_decode_attention_workspace_bytes(int nh, int max_pos) {
  if (nh < 1 || max_pos < 1) return 0;
  return bp::decode_attention_workspace_bytes(nh, max_pos);
}

extern "C" int bp_decode_attention(const void* qkv, const void* q_norm_w, const void* k_norm_w, const float* cos_t,
                                   const float* sin_t, const int64_t* pos, void* k_cache, void* v_cache, void* out,
                                   int nh, int head_dim, int max_pos, float eps, float scale, void* workspace,
                                   size_t workspace_bytes, void* stream) {
  using namespace bp;
  clear_error();
  if (head_dim != kHd) return fail(BP_ERR_UNSUPPORTED, "decode attention supports head_dim 128 (got %d)", head_dim);
  if (nh < 1 || nh > 65535 || max_pos < 1) return fail(BP_ERR_INVALID_ARGUMENT, "bad nh=%d or max_pos=%d", nh, max_pos);
  if (qkv == nullptr || q_norm_w == nullptr || k_norm_w == nullptr || cos_t == nullptr || sin_t == nullptr ||
      pos == nullptr || k_cache == nullptr || v_cache == nullptr || out == nullptr || workspace == nullptr)
    return fail(BP_ERR_INVALID_ARGUMENT, "a pointer argument is NULL");
  if (workspace_bytes < decode_attention_workspace_bytes(nh, max_pos))
    return fail(BP_ERR_INVALID_ARGUMENT, "workspace too small (%zu < %zu bytes)", workspace_bytes,
                decode_attention_workspace_bytes(nh, max_pos));
  if (!aligned16(qkv) || !aligned16(k_cache) || !aligned16(v_cache) || !aligned16(workspace))
    return fail(BP_ERR_MISALIGNED, "qkv, the caches and the workspace must be 16-byte aligned");
  int st = require_sm100();
  if (st != BP_OK) return st;
  const int max_chunks = (max_pos + kChunk - 1) / kChunk;
  const size_t part_bytes = static_cast<size_t>(nh) * max_chunks * (kHd + 2) * sizeof(float);
  AttnArgs a{static_cast<const __nv_bfloat16*>(qkv), static_cast<const __nv_bfloat16*>(q_norm_w),
             static_cast<const __nv_bfloat16*>(k_norm_w), cos_t, sin_t, reinterpret_cast<const long long*>(pos),
             static_cast<__nv_bfloat16*>(k_cache), static_cast<__nv_bfloat16*>(v_cache),
             static_cast<__nv_bfloat16*>(out), static_cast<float*>(workspace),
             reinterpret_cast<unsigned*>(static_cast<char*>(workspace) + ((part_bytes + 255) / 256) * 256), nh, max_pos,
             max_chunks, eps, scale};
  const cudaError_t e = launch_pdl(decode_attention_kernel, dim3(max_chunks, nh), dim3(kAttnThreads),
                                   static_cast<cudaStream_t>(stream), a);
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
