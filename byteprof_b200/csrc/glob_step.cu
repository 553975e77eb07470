// One global-model step of the batch-1 byte decoder in a single persistent kernel: the OLMo-2 blocks of a
// Bolmo-1B-shaped model (d 2048, 16 heads x 128, SwiGLU 8192) at one patch position.
//
// Reference: GlobalStep.step of byteprof's minimal Bolmo loop (byteprof/optim/bolmo.py:100-136), which
// runs every block as a chain of framework kernels. The same computation exists here kernel by kernel
// (skinny GEMMs and the decode.cu glue); this kernel gives the same result except for the summation order
// inside the matrix-vector products, and removes the ~8 kernel boundaries per block.
//
// Work layout. Each CTA (one per SM, cooperative launch) owns a contiguous slice of the rows of every
// weight matrix: qkv [3d, d], o [d, d], the gate and up halves of gu [2 ffn, d] (the same row indices in
// both), down [d, ffn]. Its producer warp streams these slices, block after block, in 16 KB 1-D bulk
// copies into a 12-slot shared-memory ring. Weights never depend on activations, so the stream runs ahead
// of the computation and through the grid barriers, and HBM stays busy while CTAs wait for each other.
// The 8 consumer warps run five phases per block, each ended by a grid barrier:
//   1 qkv   x = the block input (the patch vector, or h + rmsnorm(dn) * mlp_norm of the block before,
//           recomputed by every CTA from global memory); y = W_qkv x
//   2 attn  16 heads x 8 position chunks: q, k RMSNorm over d, rotary embedding, the cache write of
//           position p (the chunk that holds p), scores and a softmax partial (max, sum, output)
//   3 o     att = the 8 partials of each head merged in chunk order (every CTA); o = W_o att
//   4 gu    h = x + rmsnorm(o) * attn_norm; a = silu(W_gate h) * (W_up h)
//   5 down  dn = W_down a
// After the last block CTA 0 writes value = rmsnorm(h + rmsnorm(dn) * mlp_norm) * out_norm and advances
// the patch position. Norms, rotary embedding, softmax and SwiGLU round exactly as the decode.cu kernels.
//
// Grid barriers: one arrival counter in global memory (release add, acquire polling). A CTA that waits
// longer than kWaitLimitNs, or finds the shared abort word set, sets it (and the device error flag);
// every CTA then leaves after the bulk copies it has in flight have landed.
#include "bp_common.cuh"
#include "persist.cuh"
#include "skinny_internal.h"
#include "sm100.cuh"

namespace bp {
namespace {

using namespace persist;

constexpr int kProducers = 1;
constexpr int kThreads = threads_for(kProducers);

constexpr int kD = 2048, kNH = 16, kHd = 128, kFfn = 8192;
constexpr int kQkvRows = 3 * kD;
constexpr int kChunks = 8;                        // attention position chunks per head
constexpr int kPerWarp = 16;                      // positions per warp and round
constexpr int kSpan = kConsumerWarps * kPerWarp;  // 128 positions per chunk and round
constexpr int kRound = kChunks * kSpan;           // 1024
constexpr int kPartO = 4;                         // partial: max, sum, 2 unused, output[128] (16-byte aligned)
constexpr int kPart = kPartO + kHd;
constexpr int kRows2048 = kSlotBytes / (kD * 2);  // 4 rows of K = 2048 per slot
constexpr int kMaxLayers = 32;
constexpr int kMaxGuRows = 128;                   // gate rows per CTA (needs >= 64 CTAs)

struct Layer {
  const __nv_bfloat16 *w_qkv, *q_norm, *k_norm, *w_o, *attn_norm, *w_gu, *w_down, *mlp_norm;
  __nv_bfloat16 *kc, *vc;
};

struct Args {
  Layer L[kMaxLayers];
  int n_layers, max_pos;
  const __nv_bfloat16* x_in;
  const __nv_bfloat16* out_norm;
  __nv_bfloat16* value_out;
  long long* pos;
  const float* cos_t;
  const float* sin_t;
  float eps, scale;
  uint32_t* y;     // [3d] tagged (see st_tagged)
  float* part;     // [nh][kChunks][kPart]
  uint32_t* o;     // [d] tagged
  uint32_t* a;     // [ffn] tagged
  uint32_t* dn;    // [d] tagged
  unsigned* sync;  // [0] barrier arrivals (grows during a launch), [2] abort, [8] launch number (kept)
};

struct Smem {
  Ring r;
  alignas(16) __nv_bfloat16 vec[kFfn];  // the phase's input vector
  alignas(16) float wo[kConsumerWarps][kHd];
  alignas(16) float qs[kHd];
  alignas(16) float ks[kHd];
  alignas(16) float vs[kHd];
  float wm[kConsumerWarps], wl[kConsumerWarps];
  float gbuf[kMaxGuRows], ubuf[kMaxGuRows];  // gate and up values of this CTA's rows
};

// out[e] = bf16(res[e] + bf16(src[e] * inv * w[e])) for this thread's 8 elements e = 8 t .. 8 t + 7 of a
// d-vector, inv from the sum of squares of src (decode.cu's BP_NORM_ADD_AFTER with a 256-thread team). src
// is a tagged hand-off, res this thread's 8 values; the result goes to shared memory and to `out`. Every
// consumer reaches the CTA barrier inside, whether its wait succeeded or not; false when the step stops.
__device__ bool add_norm_tagged(const uint32_t* src, uint32_t tag, const float (&res)[8], const __nv_bfloat16* w,
                                float eps, Smem& s, float* red, unsigned* sync, float (&out)[8]) {
  const int e = threadIdx.x * 8;
  float f[8], wv[8];
  const uint4 wraw = ldg16(w + e);  // in flight during the wait (the barriers below keep later loads behind)
  const bool ok = ld_tagged8(src + e, tag, f, sync);
  float ss = 0.0f;
#pragma unroll
  for (int j = 0; j < 8; ++j) ss = fmaf(f[j], f[j], ss);
  const float inv = inv_rms(consumer_sum(ss, red), kD, eps);
  unpack8(wraw, wv);
#pragma unroll
  for (int j = 0; j < 8; ++j) out[j] = round_bf16(__fadd_rn(res[j], round_bf16(__fmul_rn(__fmul_rn(f[j], inv), wv[j]))));
  *reinterpret_cast<uint4*>(&s.vec[e]) = pack8(out);
  return ok;
}

// Row . vec for a bf16 row of 8192 in shared memory against the 8192-vector in s.vec.
__device__ __forceinline__ float dot8192(const uint8_t* row, const Smem& s) {
  const int lane = threadIdx.x & 31;
  float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll 8
  for (int i = 0; i < kFfn / 256; ++i) {
    float w[8], x[8];
    unpack8(*reinterpret_cast<const uint4*>(row + (lane * 8 + 256 * i) * 2), w);
    unpack8(*reinterpret_cast<const uint4*>(&s.vec[lane * 8 + 256 * i]), x);
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[j & 3] = fmaf(w[j], x[j], acc[j & 3]);
  }
  float v = (acc[0] + acc[1]) + (acc[2] + acc[3]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(kFull, v, o);
  return v;
}

// Rows [r0, r1) of a K = 2048 weight, in 4-row ring chunks from chunk j0: warp w takes the chunks w,
// w + 8, ... whole (one reader per chunk); out[row] = bf16(row . x), tagged. The warps run independently; a
// warp whose wait fails (the CTA stops) leaves, and the end of the phase tells the others.
__device__ uint32_t gemv2048(Smem& s, uint32_t j0, int r0, int r1, const float (&xr)[64], uint32_t* out, uint32_t tag) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nch = (r1 - r0 + kRows2048 - 1) / kRows2048;
  for (int ch = warp; ch < nch; ch += kConsumerWarps) {
    const uint8_t* slot = acquire(s.r, j0 + ch);
    if (slot == nullptr) break;
    float v[kRows2048];
    dot4x2048(slot, xr, v);
    release(s.r, j0 + ch, 1);
    if (lane < kRows2048 && r0 + ch * kRows2048 + lane < r1) st_tagged(out + r0 + ch * kRows2048 + lane, lane_row(v), tag);
  }
  return j0 + nch;
}

// ---- the producer: this CTA's weight slices, in the consumers' order --------------------------------
// Chunk k of this CTA's stream (the same sequence for every block): the qkv rows in 4-row chunks, the o
// rows in 4-row chunks, the gate rows in 4-row chunks, the same up rows in 4-row chunks (two contiguous
// runs: 574 us per step against 585 with gate and up chunks alternating), then the down rows one per chunk.
struct Stream {
  int q0, q1, o0, o1, g0, g1, d0, d1;  // this CTA's row ranges
  int nq, no, ng, nd, per_layer;       // chunks per segment and per block
  __device__ Stream(int c, int G) {
    split(kQkvRows, G, c, q0, q1);
    split(kD, G, c, o0, o1);
    split(kFfn, G, c, g0, g1);
    split(kD, G, c, d0, d1);
    nq = (q1 - q0 + kRows2048 - 1) / kRows2048;
    no = (o1 - o0 + kRows2048 - 1) / kRows2048;
    ng = 2 * ((g1 - g0 + kRows2048 - 1) / kRows2048);
    nd = d1 - d0;
    per_layer = nq + no + ng + nd;
  }
  __device__ const void* chunk(const Args& a, int k, uint32_t& bytes) const {
    const Layer& L = a.L[k / per_layer];
    int i = k % per_layer;
    if (i < nq) {
      const int r = q0 + i * kRows2048;
      bytes = min(kRows2048, q1 - r) * kD * 2;
      return L.w_qkv + static_cast<size_t>(r) * kD;
    }
    i -= nq;
    if (i < no) {
      const int r = o0 + i * kRows2048;
      bytes = min(kRows2048, o1 - r) * kD * 2;
      return L.w_o + static_cast<size_t>(r) * kD;
    }
    i -= no;
    if (i < ng) {
      const int up = i >= ng / 2 ? 1 : 0;
      const int r = g0 + (i - up * (ng / 2)) * kRows2048;
      bytes = min(kRows2048, g1 - r) * kD * 2;
      return L.w_gu + static_cast<size_t>(up * kFfn + r) * kD;
    }
    i -= ng;
    bytes = kFfn * 2;
    return L.w_down + static_cast<size_t>(d0 + i) * kFfn;
  }
};

struct StreamSrc {
  const Args& a;
  Stream st;
  __device__ const void* chunk(int k, uint32_t& bytes) const { return st.chunk(a, k, bytes); }
};

// ---- phase 2: one (head, chunk) unit of the attention ---------------------------------------------------
// A (head, chunk) unit has work when one of its positions is at most p: chunk c covers the positions
// c kSpan + r kRound + [0, kSpan) of rounds r = 0 .. p / kRound. Units without any (c kSpan > p < kRound)
// neither run nor write a partial; the merge skips their chunks (a partial of no position contributed
// exactly nothing: m = -inf, weight 0).
__device__ __forceinline__ bool chunk_active(int chunk, long long p) {
  return p >= kRound || static_cast<long long>(chunk) * kSpan <= p;
}

// Requests into L2 the cache rows (k and v, head h) that unit (h, chunk) will read: the positions below p,
// written by earlier steps, so the request can go out at the start of the block.
__device__ void prefetch_unit_rows(const Layer& L, int h, int chunk, long long p) {
  const int tid = threadIdx.x;
  const int rounds = static_cast<int>(p / kRound) + 1;
  for (int r = 0; r < rounds; ++r) {
    const long long pos = static_cast<long long>(r) * kRound + chunk * kSpan + (tid >> 1);
    if (tid < 2 * kSpan && pos < p) {
      const long long off = (pos * kNH + h) * kHd + (tid & 1) * (kHd / 2);  // one 128-byte half of the row
      asm volatile("prefetch.global.L2 [%0];" ::"l"(L.kc + off));
      asm volatile("prefetch.global.L2 [%0];" ::"l"(L.vc + off));
    }
  }
}

// q, k, v come from the tagged hand-off y (tag `tag`); false when the step stops (every consumer still
// reaches the CTA barriers inside).
__device__ bool attention_unit(const Args& a, Smem& s, const Layer& L, int h, int chunk, long long p, uint32_t tag) {
  constexpr int kHalf = kHd / 2;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int rounds = static_cast<int>(p / kRound) + 1;
  const bool own = static_cast<int>((p % kRound) / kSpan) == chunk;
  const uint32_t* q = a.y;
  const uint32_t* k = a.y + kD;
  const uint32_t* v = a.y + 2 * kD;
  bool ok = true;
  auto load_rows = [&](long long base, uint2 (&kk)[kPerWarp], uint2 (&vv)[kPerWarp]) {
#pragma unroll
    for (int j = 0; j < kPerWarp; ++j) {
      kk[j] = make_uint2(0u, 0u);
      vv[j] = make_uint2(0u, 0u);
      if (base + j < p) {  // rows below p were written by earlier steps; row p comes from this unit
        const long long off = ((base + j) * kNH + h) * kHd + lane * 4;
        kk[j] = __ldg(reinterpret_cast<const uint2*>(L.kc + off));
        vv[j] = __ldg(reinterpret_cast<const uint2*>(L.vc + off));
      }
    }
  };
  uint2 kk[kPerWarp], vv[kPerWarp];
  load_rows(static_cast<long long>(chunk) * kSpan + warp * kPerWarp, kk, vv);
  const int hi = h * kHd + (tid % kHalf);
  float cs = 0.0f, sn = 0.0f, qa = 0.0f, qb = 0.0f, qwa = 0.0f, qwb = 0.0f, ka = 0.0f, kb = 0.0f, kwa = 0.0f, kwb = 0.0f;
  float va = 0.0f, vb = 0.0f;
  // the rotary factors and norm weights first (they do not wait for y), then every load of y this thread
  // needs in flight at once, then the tag checks: this thread's 8 values of q and k (for the norms over d),
  // and its rotary pair of q, k and its v pair of this head
  if (tid < kHalf) {
    cs = a.cos_t[p * kHalf + tid];
    sn = a.sin_t[p * kHalf + tid];
    qwa = __bfloat162float(L.q_norm[hi]);
    qwb = __bfloat162float(L.q_norm[hi + kHalf]);
    if (own) {
      kwa = __bfloat162float(L.k_norm[hi]);
      kwb = __bfloat162float(L.k_norm[hi + kHalf]);
    }
  }
  const uint4 q0 = ld_relaxed16(q + tid * 8), q1 = ld_relaxed16(q + tid * 8 + 4);
  const uint4 k0 = ld_relaxed16(k + tid * 8), k1 = ld_relaxed16(k + tid * 8 + 4);
  const int vj = h * kHd + (tid - kHalf) * 2;
  const bool rot = tid < kHalf, vown = !rot && own && tid < kHd;
  uint32_t w0 = 0, w1 = 0, w2 = 0, w3 = 0;
  if (rot) {
    w0 = ld_relaxed4(q + hi);
    w1 = ld_relaxed4(q + hi + kHalf);
    if (own) {
      w2 = ld_relaxed4(k + hi);
      w3 = ld_relaxed4(k + hi + kHalf);
    }
  } else if (vown) {
    w0 = ld_relaxed4(v + vj);
    w1 = ld_relaxed4(v + vj + 1);
  }
  float fq[8], fk[8];
  ok &= take_tagged8(q0, q1, q + tid * 8, tag, fq, a.sync);
  ok &= take_tagged8(k0, k1, k + tid * 8, tag, fk, a.sync);
  if (rot) {
    ok &= take_tagged1(w0, q + hi, tag, qa, a.sync);
    ok &= take_tagged1(w1, q + hi + kHalf, tag, qb, a.sync);
    if (own) {
      ok &= take_tagged1(w2, k + hi, tag, ka, a.sync);
      ok &= take_tagged1(w3, k + hi + kHalf, tag, kb, a.sync);
    }
  } else if (vown) {
    ok &= take_tagged1(w0, v + vj, tag, va, a.sync);
    ok &= take_tagged1(w1, v + vj + 1, tag, vb, a.sync);
  }
  float sq = 0.0f, sk = 0.0f;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    sq = fmaf(fq[j], fq[j], sq);
    sk = fmaf(fk[j], fk[j], sk);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    sq += __shfl_xor_sync(kFull, sq, o);
    sk += __shfl_xor_sync(kFull, sk, o);
  }
  if (lane == 0) {
    s.r.red[0][warp] = sq;
    s.r.red[1][warp] = sk;
  }
  consumer_sync();
  float tq = 0.0f, tk = 0.0f;
#pragma unroll
  for (int w = 0; w < kConsumerWarps; ++w) {
    tq += s.r.red[0][w];
    tk += s.r.red[1][w];
  }
  const float inv_q = inv_rms(tq, kD, a.eps), inv_k = inv_rms(tk, kD, a.eps);
  const long long slot = p * kNH + h;
  if (tid < kHalf) {
    const float q0 = round_bf16(__fmul_rn(__fmul_rn(qa, inv_q), qwa));
    const float q1 = round_bf16(__fmul_rn(__fmul_rn(qb, inv_q), qwb));
    s.qs[tid] = __fsub_rn(__fmul_rn(q0, cs), __fmul_rn(q1, sn));
    s.qs[tid + kHalf] = __fadd_rn(__fmul_rn(q1, cs), __fmul_rn(q0, sn));
    if (own) {
      const float k0 = round_bf16(__fmul_rn(__fmul_rn(ka, inv_k), kwa));
      const float k1 = round_bf16(__fmul_rn(__fmul_rn(kb, inv_k), kwb));
      const __nv_bfloat16 r0 = __float2bfloat16_rn(__fsub_rn(__fmul_rn(k0, cs), __fmul_rn(k1, sn)));
      const __nv_bfloat16 r1 = __float2bfloat16_rn(__fadd_rn(__fmul_rn(k1, cs), __fmul_rn(k0, sn)));
      L.kc[slot * kHd + tid] = r0;
      L.kc[slot * kHd + tid + kHalf] = r1;
      s.ks[tid] = __bfloat162float(r0);
      s.ks[tid + kHalf] = __bfloat162float(r1);
    }
  } else if (own && tid < kHd) {
    const int j = (tid - kHalf) * 2;
    L.vc[slot * kHd + j] = __float2bfloat16_rn(va);
    L.vc[slot * kHd + j + 1] = __float2bfloat16_rn(vb);
    s.vs[j] = va;
    s.vs[j + 1] = vb;
  }
  consumer_sync();

  const float4 qv = *reinterpret_cast<const float4*>(&s.qs[lane * 4]);
  float mw = -INFINITY, lw = 0.0f, o4[4] = {0.0f, 0.0f, 0.0f, 0.0f};
  for (int r = 0; r < rounds; ++r) {
    const long long base = static_cast<long long>(r) * kRound + chunk * kSpan + warp * kPerWarp;
    if (r > 0) load_rows(base, kk, vv);
    float sc[kPerWarp];
#pragma unroll
    for (int j = 0; j < kPerWarp; ++j) {
      float k4[4];
      if (base + j == p) {
        const float4 t = *reinterpret_cast<const float4*>(&s.ks[lane * 4]);
        k4[0] = t.x; k4[1] = t.y; k4[2] = t.z; k4[3] = t.w;
      } else {
        k4[0] = bf16lo(kk[j].x); k4[1] = bf16hi(kk[j].x); k4[2] = bf16lo(kk[j].y); k4[3] = bf16hi(kk[j].y);
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
    if (mr == -INFINITY) continue;
    const float m_new = fmaxf(mw, mr);
    if (mw != -INFINITY) {
      const float f = expf(__fsub_rn(mw, m_new));
      lw = __fmul_rn(lw, f);
#pragma unroll
      for (int cc = 0; cc < 4; ++cc) o4[cc] = __fmul_rn(o4[cc], f);
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
        const float4 t = *reinterpret_cast<const float4*>(&s.vs[lane * 4]);
        v4[0] = t.x; v4[1] = t.y; v4[2] = t.z; v4[3] = t.w;
      } else {
        v4[0] = bf16lo(vv[j].x); v4[1] = bf16hi(vv[j].x); v4[2] = bf16lo(vv[j].y); v4[3] = bf16hi(vv[j].y);
      }
#pragma unroll
      for (int cc = 0; cc < 4; ++cc) o4[cc] = fmaf(e[j], v4[cc], o4[cc]);
    }
  }
  if (lane == 0) {
    s.wm[warp] = mw;
    s.wl[warp] = lw;
  }
  *reinterpret_cast<float4*>(&s.wo[warp][lane * 4]) = make_float4(o4[0], o4[1], o4[2], o4[3]);
  consumer_sync();
  if (tid < kHd) {
    float mc = -INFINITY;
#pragma unroll
    for (int w = 0; w < kConsumerWarps; ++w) mc = fmaxf(mc, s.wm[w]);
    float lc = 0.0f, oc = 0.0f;
    if (mc != -INFINITY) {
#pragma unroll
      for (int w = 0; w < kConsumerWarps; ++w) {
        const float f = s.wm[w] == -INFINITY ? 0.0f : expf(__fsub_rn(s.wm[w], mc));
        lc = fmaf(s.wl[w], f, lc);
        oc = fmaf(s.wo[w][tid], f, oc);
      }
    }
    float* pc = a.part + (static_cast<long long>(h) * kChunks + chunk) * kPart;
    pc[kPartO + tid] = oc;
    if (tid == 0) {
      pc[0] = mc;
      pc[1] = lc;
    }
  }
  consumer_sync();  // shared scratch is reused by the next unit
  return ok;
}

// ---- the consumers --------------------------------------------------------------------------------------
// Hand-offs of block l (tags hand_tag(seq, 4 l + i)): i = 0 y (qkv -> attention), 1 o (-> gate/up),
// 2 a (-> down), 3 dn (-> the next block's qkv, or the final norm), each after a grid barrier without fence,
// except y: only the (at most 128) active attention units read it, and they poll its words directly (557
// against 571 us per step with the signal).
// The partials of the attention go to the o phase through an ordered grid barrier (its fence is cheap
// there: the ring is full and no copy is in flight).
// Every CTA computes the block input x and the residual h itself and keeps its 8 values per thread.
__device__ void consumers(const Args& a, Smem& s, int c, int G, long long p, unsigned seq) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  unsigned epoch = 0;  // grid barriers passed (thread 0)
  uint32_t j = 0;  // ring chunk counter, in the producer's order
  float xr[64];
  float xreg[8], hreg[8];  // x and h at elements 8 tid .. 8 tid + 7
  for (int l = 0; l < a.n_layers; ++l) {
    const Layer& L = a.L[l];
    const uint32_t tag_y = hand_tag(seq, 4 * l), tag_o = hand_tag(seq, 4 * l + 1), tag_a = hand_tag(seq, 4 * l + 2),
                   tag_dn = hand_tag(seq, 4 * l + 3);
    // ---- 1: x and y = W_qkv x
    bool ok = true;
    if (l == 0) {
      const uint4 xv = ldg16(a.x_in + tid * 8);
      unpack8(xv, xreg);
      *reinterpret_cast<uint4*>(&s.vec[tid * 8]) = xv;
    } else {
      ok = add_norm_tagged(a.dn, hand_tag(seq, 4 * l - 1), hreg, a.L[l - 1].mlp_norm, a.eps, s, s.r.red[0], a.sync,
                           xreg);
    }
    if (consumers_stop_if(s.r, a.sync, !ok)) return;  // also the CTA barrier after s.vec
    for (int u = c; u < kNH * kChunks; u += G)
      if (chunk_active(u % kChunks, p)) prefetch_unit_rows(L, u / kChunks, u % kChunks, p);
    load_lane_x(s.vec, xr);
    int r0, r1;
    split(kQkvRows, G, c, r0, r1);
    j = gemv2048(s, j, r0, r1, xr, a.y, tag_y);
    if (consumers_stop(s.r, a.sync)) return;
    // ---- 2: attention (the active units wait for y word by word: no signal)
    ok = true;
    for (int u = c; u < kNH * kChunks; u += G)
      if (chunk_active(u % kChunks, p)) ok &= attention_unit(a, s, L, u / kChunks, u % kChunks, p, tag_y);
    if (consumers_stop_if(s.r, a.sync, !ok) || !grid_sync(s.r, a.sync, epoch)) return;
    // ---- 3: att (merge of the partials) and o = W_o att
    {
      const int e = tid * 8, h = e / kHd, dd = e % kHd;
      const float* ph = a.part + static_cast<long long>(h) * kChunks * kPart;
      float mc[kChunks], mg = -INFINITY;
#pragma unroll
      for (int ch = 0; ch < kChunks; ++ch) {
        mc[ch] = chunk_active(ch, p) ? __ldcg(ph + ch * kPart) : -INFINITY;
        mg = fmaxf(mg, mc[ch]);
      }
      float lg = 0.0f, og[8] = {0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
      for (int ch = 0; ch < kChunks; ++ch) {
        if (!chunk_active(ch, p)) continue;
        const float f = mc[ch] == -INFINITY ? 0.0f : expf(__fsub_rn(mc[ch], mg));
        lg = fmaf(__ldcg(ph + ch * kPart + 1), f, lg);
        const float4 o0 = __ldcg(reinterpret_cast<const float4*>(ph + ch * kPart + kPartO + dd));
        const float4 o1 = __ldcg(reinterpret_cast<const float4*>(ph + ch * kPart + kPartO + dd + 4));
        const float ov[8] = {o0.x, o0.y, o0.z, o0.w, o1.x, o1.y, o1.z, o1.w};
#pragma unroll
        for (int i = 0; i < 8; ++i) og[i] = fmaf(ov[i], f, og[i]);
      }
      float at[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) at[i] = __fdiv_rn(og[i], lg);
      *reinterpret_cast<uint4*>(&s.vec[e]) = make_uint4(pack_bf16x2(at[0], at[1]), pack_bf16x2(at[2], at[3]),
                                                        pack_bf16x2(at[4], at[5]), pack_bf16x2(at[6], at[7]));
    }
    consumer_sync();
    load_lane_x(s.vec, xr);
    split(kD, G, c, r0, r1);
    j = gemv2048(s, j, r0, r1, xr, a.o, tag_o);
    if (consumers_stop(s.r, a.sync) || !grid_sync(s.r, a.sync, epoch, false)) return;
    // ---- 4: h = x + rmsnorm(o) * attn_norm; a = silu(W_gate h) * (W_up h)
    ok = add_norm_tagged(a.o, tag_o, xreg, L.attn_norm, a.eps, s, s.r.red[0], a.sync, hreg);
    if (consumers_stop_if(s.r, a.sync, !ok)) return;
    load_lane_x(s.vec, xr);
    split(kFfn, G, c, r0, r1);
    {
      // chunk m < npairs: gate rows r0 + 4m .., chunk npairs + m: the same up rows; warp w takes the
      // chunks w, w + 8, ... whole
      const int npairs = (r1 - r0 + kRows2048 - 1) / kRows2048;
      for (int ch = warp; ch < 2 * npairs; ch += kConsumerWarps) {
        const uint8_t* slot = acquire(s.r, j + ch);
        if (slot == nullptr) break;
        float v[kRows2048];
        dot4x2048(slot, xr, v);
        release(s.r, j + ch, 1);
        const bool up = ch >= npairs;
        const int rl = (up ? ch - npairs : ch) * kRows2048 + lane;
        if (lane < kRows2048 && r0 + rl < r1) (up ? s.ubuf : s.gbuf)[rl] = lane_row(v);
      }
      j += 2 * npairs;
    }
    if (consumers_stop(s.r, a.sync)) return;
    for (int rl = tid; rl < r1 - r0; rl += kConsumers) {
      const float g = round_bf16(s.gbuf[rl]), up = round_bf16(s.ubuf[rl]);
      const float sl = round_bf16(static_cast<float>(g / (1.0 + exp(-static_cast<double>(g)))));
      st_tagged(a.a + r0 + rl, __fmul_rn(sl, up), tag_a);
    }
    if (!grid_sync(s.r, a.sync, epoch, false)) return;
    // ---- 5: dn = W_down a
    ok = true;
    {
      constexpr int kGroups = kFfn / (kConsumers * 8);
      uint4 ua[kGroups][2];  // all loads in flight, then the tag checks
#pragma unroll
      for (int i = 0; i < kGroups; ++i) {
        const uint32_t* pa = a.a + (i * kConsumers + tid) * 8;
        ua[i][0] = ld_relaxed16(pa);
        ua[i][1] = ld_relaxed16(pa + 4);
      }
#pragma unroll
      for (int i = 0; i < kGroups; ++i) {
        const int e = (i * kConsumers + tid) * 8;
        float f[8];
        ok &= take_tagged8(ua[i][0], ua[i][1], a.a + e, tag_a, f, a.sync);
        *reinterpret_cast<uint4*>(&s.vec[e]) = pack8(f);
      }
    }
    if (consumers_stop_if(s.r, a.sync, !ok)) return;
    split(kD, G, c, r0, r1);
    for (int q = warp; q < r1 - r0; q += kConsumerWarps) {  // one row per chunk, one reader warp
      const uint8_t* slot = acquire(s.r, j + q);
      if (slot == nullptr) break;
      const float v = dot8192(slot, s);
      if (lane == 0) st_tagged(a.dn + r0 + q, v, tag_dn);
      release(s.r, j + q, 1);
    }
    j += r1 - r0;
    if (consumers_stop(s.r, a.sync) || !grid_sync(s.r, a.sync, epoch, false)) return;
  }
  // ---- value = rmsnorm(x_L) * out_norm, x_L = h + rmsnorm(dn) * mlp_norm of the last block
  if (c != 0) return;
  const int last = a.n_layers - 1;
  const uint4 onw = ldg16(a.out_norm + tid * 8);  // before the waits
  float xl[8];
  const bool ok = add_norm_tagged(a.dn, hand_tag(seq, 4 * last + 3), hreg, a.L[last].mlp_norm, a.eps, s, s.r.red[0],
                                  a.sync, xl);
  if (consumers_stop_if(s.r, a.sync, !ok)) return;
  const int e = tid * 8;
  float wv[8];
  float ss = 0.0f;
#pragma unroll
  for (int i = 0; i < 8; ++i) ss = fmaf(xl[i], xl[i], ss);
  const float inv = inv_rms(consumer_sum(ss, s.r.red[1]), kD, a.eps);
  unpack8(onw, wv);
  float o[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) o[i] = __fmul_rn(__fmul_rn(xl[i], inv), wv[i]);
  *reinterpret_cast<uint4*>(a.value_out + e) = pack8(o);
  if (tid == 0) *a.pos = p + 1;
}

__global__ void __launch_bounds__(kThreads, 1) glob_step_kernel(Args a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  Smem& s = *reinterpret_cast<Smem*>(smem_raw);
  const int c = blockIdx.x, G = gridDim.x;
  const long long p = *a.pos;
  const bool valid = p >= 0 && p < a.max_pos;  // the same answer in every CTA
  if (threadIdx.x == 0) ring_init(s.r);
  __syncthreads();
  if (threadIdx.x >= kConsumers) {
    if ((threadIdx.x & 31) == 0) {
      const StreamSrc src{a, Stream(c, G)};
      produce<kProducers>(s.r, src, valid ? src.st.per_layer * a.n_layers : 0, (threadIdx.x - kConsumers) / 32);
    }
    return;
  }
  if (!valid) {  // host checks keep p in range; never index with a bad one
    if (c == 0) {
      const uint4 nan4 = make_uint4(0x7fc07fc0u, 0x7fc07fc0u, 0x7fc07fc0u, 0x7fc07fc0u);
      *reinterpret_cast<uint4*>(a.value_out + threadIdx.x * 8) = nan4;
    }
    return;
  }
  const unsigned seq = *reinterpret_cast<volatile unsigned*>(a.sync + 8);  // this launch's number (tags)
  consumers(a, s, c, G, p, seq);
  // CTA 0 finishes last (it reads every CTA's last output); every CTA read the number at its start
  if (c == 0 && threadIdx.x == 0) *reinterpret_cast<volatile unsigned*>(a.sync + 8) = seq + 1;
}

constexpr size_t kWsY = 0;  // tagged hand-offs: 4 bytes per value
constexpr size_t kWsPart = kWsY + 3 * kD * 4;
constexpr size_t kWsO = kWsPart + static_cast<size_t>(kNH) * kChunks * kPart * 4;
constexpr size_t kWsA = kWsO + kD * 4;
constexpr size_t kWsDn = kWsA + kFfn * 4;
constexpr size_t kWsSync = kWsDn + kD * 4;
constexpr size_t kWsBytes = kWsSync + 256;

}  // namespace

BP_DEFINE_DEVICE_ERROR_READER(read_device_errors_glob)

}  // namespace bp

extern "C" size_t bp_glob_step_workspace_bytes(void) { return bp::kWsBytes; }

extern "C" int bp_glob_step(const bp_glob_layer* layers, int n_layers, const void* x_in, const void* out_norm,
                            void* value_out, int64_t* pos, const float* cos_t, const float* sin_t, int max_pos,
                            float eps, void* workspace, size_t workspace_bytes, void* stream) {
  using namespace bp;
  clear_error();
  if (layers == nullptr || n_layers < 1 || n_layers > kMaxLayers)
    return fail(BP_ERR_INVALID_ARGUMENT, "need 1..%d layers (got %d)", kMaxLayers, n_layers);
  if (x_in == nullptr || out_norm == nullptr || value_out == nullptr || pos == nullptr || cos_t == nullptr ||
      sin_t == nullptr || workspace == nullptr || max_pos < 1)
    return fail(BP_ERR_INVALID_ARGUMENT, "a pointer argument is NULL or max_pos < 1");
  if (workspace_bytes < kWsBytes)
    return fail(BP_ERR_INVALID_ARGUMENT, "workspace too small (%zu < %zu bytes)", workspace_bytes, kWsBytes);
  auto a16 = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15u) == 0; };
  if (!a16(x_in) || !a16(out_norm) || !a16(value_out) || !a16(workspace))
    return fail(BP_ERR_MISALIGNED, "vectors and the workspace must be 16-byte aligned");
  Args a{};
  for (int l = 0; l < n_layers; ++l) {
    const bp_glob_layer& g = layers[l];
    const void* ptrs[] = {g.w_qkv, g.q_norm, g.k_norm, g.w_o, g.attn_norm, g.w_gu, g.w_down, g.mlp_norm, g.k_cache,
                          g.v_cache};
    for (const void* q : ptrs)
      if (q == nullptr || !a16(q)) return fail(BP_ERR_MISALIGNED, "layer %d: a NULL or unaligned pointer", l);
    a.L[l] = Layer{static_cast<const __nv_bfloat16*>(g.w_qkv), static_cast<const __nv_bfloat16*>(g.q_norm),
                   static_cast<const __nv_bfloat16*>(g.k_norm), static_cast<const __nv_bfloat16*>(g.w_o),
                   static_cast<const __nv_bfloat16*>(g.attn_norm), static_cast<const __nv_bfloat16*>(g.w_gu),
                   static_cast<const __nv_bfloat16*>(g.w_down), static_cast<const __nv_bfloat16*>(g.mlp_norm),
                   static_cast<__nv_bfloat16*>(g.k_cache), static_cast<__nv_bfloat16*>(g.v_cache)};
  }
  a.n_layers = n_layers;
  a.max_pos = max_pos;
  a.x_in = static_cast<const __nv_bfloat16*>(x_in);
  a.out_norm = static_cast<const __nv_bfloat16*>(out_norm);
  a.value_out = static_cast<__nv_bfloat16*>(value_out);
  a.pos = reinterpret_cast<long long*>(pos);
  a.cos_t = cos_t;
  a.sin_t = sin_t;
  a.eps = eps;
  a.scale = 1.0f / sqrtf(static_cast<float>(kHd));
  char* ws = static_cast<char*>(workspace);
  a.y = reinterpret_cast<uint32_t*>(ws + kWsY);
  a.part = reinterpret_cast<float*>(ws + kWsPart);
  a.o = reinterpret_cast<uint32_t*>(ws + kWsO);
  a.a = reinterpret_cast<uint32_t*>(ws + kWsA);
  a.dn = reinterpret_cast<uint32_t*>(ws + kWsDn);
  a.sync = reinterpret_cast<unsigned*>(ws + kWsSync);
  int st = require_sm100();
  if (st != BP_OK) return st;
  const size_t smem = sizeof(Smem);
  cudaError_t e = cudaFuncSetAttribute(glob_step_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return fail(BP_ERR_CUDA, "glob_step smem attribute: %s", cudaGetErrorString(e));
  const int sms = tc_sm_count();
  if ((kFfn + sms - 1) / sms > kMaxGuRows) return fail(BP_ERR_UNSUPPORTED, "glob_step needs at least 64 SMs");
  int per_sm = 0;
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, glob_step_kernel, kThreads, smem);
  if (e != cudaSuccess || per_sm < 1) return fail(BP_ERR_CUDA, "glob_step does not fit on an SM");
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  e = cudaMemsetAsync(a.sync, 0, 16, s);  // arrival counter, abort word (the launch number stays)
  if (e != cudaSuccess) return fail(BP_ERR_CUDA, "glob_step sync reset: %s", cudaGetErrorString(e));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(sms);  // one CTA per SM, all resident (cooperative launch)
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, glob_step_kernel, a);
  if (e != cudaSuccess) return fail(BP_ERR_CUDA, "glob_step launch: %s", cudaGetErrorString(e));
  return check_launch("glob_step");
}
