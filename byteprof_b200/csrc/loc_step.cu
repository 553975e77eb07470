// One local (byte-level) step of the batch-1 byte decoder in a single persistent kernel, for the
// Bolmo-shaped local layers (d 2048, mLSTM 4 heads x 512, SwiGLU 2816, byte vocabulary 512):
//   encoder: h = embed[byte]; one mLSTM layer; e = rmsnorm(layer output) * enc_norm;
//            patch = W_patch e; boundary logit = w_boundary . e (fp32)
//   decoder: h = W_in e + value; one mLSTM layer; logits = LM head (rmsnorm(layer output) * final_norm)
//            (fp32); out = [argmax(logits), sigmoid(boundary logit) >= 0.5]
//   both (a byte that opens no patch): the encoder step, then the decoder step on its e and boundary logit,
//            in one launch: one ring stream and one barrier sequence over both parts
// The layer: x = rmsnorm(h) * norm1; y = W_qkvo x (q | k | v | o), g = cap * tanh((W_if x + b_if) / cap);
// the mLSTM step (state C in place, n / m from buffer `cur` to buffer `next`); z = sigmoid(o) *
// rmsnorm_head(h_mlstm) * mh_norm; h2 = h + W_out z; a = silu(W_gate x2) * (W_up x2) with
// x2 = rmsnorm(h2) * norm2; layer output = h2 + W_down a.
//
// Reference: the encoder / decoder pieces of byteprof's minimal Bolmo loop (byteprof/optim/bolmo.py:32-97,
// bolmo_loop.py:36-64: _layer_step, LocalLoop.enc_step / dec_step, MinimalPieces), which run these as a
// chain of framework kernels; here the same computation is also available kernel by kernel
// (bolmo_local.LocalLayer.step), and this kernel gives the same result except for summation orders.
//
// Layout and machinery as glob_step.cu (persist.cuh): one CTA per SM, each owning row slices of every
// weight, streamed through the shared-memory ring; phases between grid barriers; every phase input is
// recomputed by every CTA from the small vectors in global memory. The mLSTM phase splits the state into
// 128 units (head, 16 value columns); each unit recomputes the head's gates and n (as the scan kernel does)
// and follows the scan kernel's precision model (bf16 gates, products and C for the output sums).
#include "bp_common.cuh"
#include "persist.cuh"
#include "skinny_internal.h"
#include "sm100.cuh"

namespace bp {
namespace {

using namespace persist;

constexpr int kProducers = 2;
constexpr int kThreads = threads_for(kProducers);

constexpr int kD = 2048, kNH = 4, kDh = 512, kFfn = 2816, kVocab = 512;
constexpr int kQkvoRows = 4 * kD;
constexpr int kCols = 16;                 // value columns per mLSTM unit
constexpr int kUnits = kNH * (kDh / kCols);  // 128
constexpr int kMaxGuRows = 64;            // gate rows per CTA (needs >= 44 CTAs)

struct Layer {
  const __nv_bfloat16 *norm1, *w_qkvo, *w_if;
  const float* b_if;
  const __nv_bfloat16 *mh_norm, *w_out, *norm2, *w_gu, *w_down;
  float* c;
  const float *n_cur, *m_cur;
  float *n_next, *m_next;
};

struct Args {
  Layer L;
  int decoder;
  // fused: this launch runs the encoder step (L) and then the decoder step (L2) of the same byte
  int fused;
  Layer L2;
  // encoder
  const __nv_bfloat16* embed;
  const long long* byte;
  const __nv_bfloat16* enc_norm;
  const __nv_bfloat16* w_patch;
  const __nv_bfloat16* w_boundary;
  __nv_bfloat16* e_out;
  __nv_bfloat16* patch_out;
  // decoder
  const __nv_bfloat16* e_in;
  const __nv_bfloat16* value;
  const __nv_bfloat16* w_in;
  const __nv_bfloat16* final_norm;
  const __nv_bfloat16* lm_head;
  float* logits;
  long long* out;
  float* boundary_logit;  // encoder: written; decoder: read
  float eps, cap, mlstm_eps, qk_scale;
  // workspace: the hand-offs between phases as tagged words (persist.cuh: st_tagged, st_tagged_f32)
  uint32_t* t;     // [d] decoder: W_in e
  uint32_t* y;     // [4d] q | k | v | o
  uint64_t* g;     // [2 nh] gate pre-activations (after the soft cap), fp32
  uint32_t* hm;    // [d] mLSTM output
  uint32_t* wo;    // [d] W_out z
  uint32_t* a;     // [ffn]
  uint32_t* dn;    // [d]
  uint64_t* lg;    // [vocab] decoder: the logits again, for the argmax, fp32
  unsigned* sync;  // [0] barrier arrivals, [2] abort, [8] launch number (kept)
  uint64_t* bnd;   // fused: the boundary logit, tagged, for the decoder part's decision (in the sync words)
};

// The tags of one launch's hand-offs (hand_tag(launch number, i)); y and the gates share one. A fused launch
// numbers its decoder part's hand-offs from 8; the boundary logit's hand-off is number 16 in either part.
struct Tags {
  uint32_t t, y, hm, wo, a, dn, lg, bnd;
  __device__ Tags(unsigned seq, int base)
      : t(hand_tag(seq, base)), y(hand_tag(seq, base + 1)), hm(hand_tag(seq, base + 2)), wo(hand_tag(seq, base + 3)),
        a(hand_tag(seq, base + 4)), dn(hand_tag(seq, base + 5)), lg(hand_tag(seq, base + 6)), bnd(hand_tag(seq, 16)) {}
};

// A run of this CTA's weight rows: chunks of `rpc` rows of `row_bytes` bytes; with pair_off > 0 the chunks
// alternate between rows r .. and the same rows + pair_off (gate and up rows of a SwiGLU weight).
struct Seg {
  const __nv_bfloat16* w;
  int r0, r1, row_bytes, rpc, pair_off;
  __device__ int chunks() const {
    const int n = r1 > r0 ? (r1 - r0 + rpc - 1) / rpc : 0;
    return pair_off > 0 ? 2 * n : n;
  }
  __device__ const void* chunk(int i, uint32_t& bytes) const {
    const int k = pair_off > 0 ? i / 2 : i;
    const int r = r0 + k * rpc;
    bytes = static_cast<uint32_t>(min(rpc, r1 - r) * row_bytes);
    const int row = r + ((pair_off > 0 && (i & 1)) ? pair_off : 0);
    return reinterpret_cast<const char*>(w) + static_cast<size_t>(row) * row_bytes;
  }
};

enum SegId { kSegIn, kSegQkvo, kSegIf, kSegOut, kSegGu, kSegDown, kSegHead, kSegBnd, kSegCount };

// This CTA's segments, in stream order (the producer's order and the consumers'). One copy per CTA in shared
// memory, built by one thread: built by every thread it went to local memory (320 copies), which the small
// L1 left beside this kernel's shared memory pushed out to L2, and the first weight copy left ~5 us after the
// kernel started.
struct Plan {
  Seg seg[kSegCount];
  int order[kSegCount], n;
  __device__ void init(const Args& a, int c, int G) {
    auto rows = [&](int id, const __nv_bfloat16* w, int nrows, int row_bytes, int rpc, int pair_off) {
      Seg& s = seg[id];
      s.w = w;
      split(nrows, G, c, s.r0, s.r1);
      s.row_bytes = row_bytes;
      s.rpc = rpc;
      s.pair_off = pair_off;
    };
    auto one = [&](int id, const __nv_bfloat16* w, int row, bool mine) {
      Seg& s = seg[id];
      s.w = w;
      s.r0 = row;
      s.r1 = mine ? row + 1 : row;
      s.row_bytes = kD * 2;
      s.rpc = 1;
      s.pair_off = 0;
    };
    for (int i = 0; i < kSegCount; ++i) seg[i] = Seg{nullptr, 0, 0, kD * 2, 1, 0};
    rows(kSegIn, a.w_in, kD, kD * 2, 4, 0);
    rows(kSegQkvo, a.L.w_qkvo, kQkvoRows, kD * 2, 4, 0);
    one(kSegIf, a.L.w_if, c, c < 2 * kNH);  // gate row c on CTA c
    rows(kSegOut, a.L.w_out, kD, kD * 2, 4, 0);
    rows(kSegGu, a.L.w_gu, kFfn, kD * 2, 4, kFfn);
    rows(kSegDown, a.L.w_down, kD, kFfn * 2, 2, 0);
    rows(kSegHead, a.decoder ? a.lm_head : a.w_patch, a.decoder ? kVocab : kD, kD * 2, 4, 0);
    one(kSegBnd, a.w_boundary, 0, !a.decoder && c == G - 1);  // the boundary row on the last CTA
    n = 0;
    if (a.decoder) order[n++] = kSegIn;
    order[n++] = kSegQkvo;
    order[n++] = kSegIf;
    order[n++] = kSegOut;
    order[n++] = kSegGu;
    order[n++] = kSegDown;
    order[n++] = kSegHead;
    if (!a.decoder) order[n++] = kSegBnd;
    index();
  }
  int first[kSegCount + 1];  // chunk number of the first chunk of stream segment i (i in stream order)
  __device__ void index() {    // once, after the segments are set: no division per chunk lookup
    first[0] = 0;
    for (int i = 0; i < n; ++i) first[i + 1] = first[i] + seg[order[i]].chunks();
  }
  __device__ int total() const { return first[n]; }
  __device__ const void* chunk(int k, uint32_t& bytes) const {
    for (int i = 0; i < n; ++i)
      if (k < first[i + 1]) return seg[order[i]].chunk(k - first[i], bytes);
    bytes = 0;
    return nullptr;
  }
};

// The producer's stream: the plan's chunks, then (fused launch) the decoder part's.
struct Stream2 {
  const Plan& p0;
  const Plan* p1;
  __device__ int total() const { return p0.total() + (p1 != nullptr ? p1->total() : 0); }
  __device__ const void* chunk(int k, uint32_t& bytes) const {
    const int t0 = p0.total();
    return k < t0 ? p0.chunk(k, bytes) : p1->chunk(k - t0, bytes);
  }
};

struct Smem {
  Ring r;
  Plan plan, plan1;  // plan1, part1: a fused launch's decoder part
  Args part1;
  alignas(16) __nv_bfloat16 vec[kD > kFfn ? kD : kFfn];  // the phase's input vector
  alignas(16) float part[kConsumerWarps][kCols];          // per-warp column sums (mLSTM unit)
  float gbuf[kMaxGuRows], ubuf[kMaxGuRows];
  float head_red[kNH][2];
  alignas(16) float kf[kDh];   // mLSTM unit: k and bf16(q * scale) of the head
  alignas(16) float qsv[kDh];
};

// ---- vector builders (all 256 consumer threads; each owns 8 elements e = 8 t .. 8 t + 7) ------------------

// This thread's 8 elements of the vectors every phase input needs that no phase writes: the norm weights
// and the layer input's own part (the embedding row, or the decoder's value and its input e), loaded at the
// start of the kernel so that no phase waits for them.
struct Pre {
  uint4 n1, n2, mh, on, h, x0;
  __device__ void load(const Args& a, long long byte) {
    const int e = threadIdx.x * 8;
    n1 = ldg16(a.L.norm1 + e);
    n2 = ldg16(a.L.norm2 + e);
    mh = ldg16(a.L.mh_norm + e);
    on = ldg16((a.decoder ? a.final_norm : a.enc_norm) + e);
    h = a.decoder ? ldg16(a.value + e) : ldg16(a.embed + byte * kD + e);
    if (a.decoder) x0 = ldg16(a.e_in + e);
  }
};

// vec = bf16(rmsnorm(src) * w) where src is a d-vector (bf16, global through L2, or given values) and w
// this thread's 8 norm weights.
__device__ void norm_into_vec(Smem& s, const float (&f)[8], uint4 w, float eps) {
  const int e = threadIdx.x * 8;
  float ss = 0.0f;
#pragma unroll
  for (int j = 0; j < 8; ++j) ss = fmaf(f[j], f[j], ss);
  const float inv = inv_rms(consumer_sum(ss, s.r.red[0]), kD, eps);
  float wv[8], o[8];
  unpack8(w, wv);
#pragma unroll
  for (int j = 0; j < 8; ++j) o[j] = __fmul_rn(__fmul_rn(f[j], inv), wv[j]);
  *reinterpret_cast<uint4*>(&s.vec[e]) = pack8(o);
}

// The layer input h (8 values of this thread): the embedding row (encoder) or bf16(W_in e + value); false
// when the step stops.
__device__ bool layer_input(const Args& a, const Tags& tg, unsigned* sy, float (&h)[8], const Pre& pre) {
  const int e = threadIdx.x * 8;
  if (!a.decoder) {
    unpack8(pre.h, h);
    return true;
  }
  float t[8], v[8];
  unpack8(pre.h, v);
  const bool ok = ld_tagged8(a.t + e, tg.t, t, sy);
#pragma unroll
  for (int j = 0; j < 8; ++j) h[j] = round_bf16(__fadd_rn(t[j], v[j]));
  return ok;
}

// h2 = bf16(h + W_out z) for this thread's 8 values; false when the step stops.
__device__ bool layer_h2(const Args& a, const Tags& tg, unsigned* sy, float (&h2)[8], const Pre& pre) {
  float h[8], w[8];
  const uint4 w0 = ld_relaxed16(a.wo + threadIdx.x * 8), w1 = ld_relaxed16(a.wo + threadIdx.x * 8 + 4);
  bool ok = layer_input(a, tg, sy, h, pre);
  ok &= take_tagged8(w0, w1, a.wo + threadIdx.x * 8, tg.wo, w, sy);
#pragma unroll
  for (int j = 0; j < 8; ++j) h2[j] = round_bf16(__fadd_rn(h[j], w[j]));
  return ok;
}

// sigmoid evaluated in double precision and rounded once (decode.cu's sigmoid_d).
__device__ __forceinline__ float sigmoid_d(float v) {
  return static_cast<float>(1.0 / (1.0 + exp(-static_cast<double>(v))));
}

// ---- GEMV phases --------------------------------------------------------------------------------------
// Output of row `row` of segment `id`: a bf16 vector, fp32 logits, a soft-capped gate or the boundary logit.
__device__ void store_row(const Args& a, const Tags& tg, int id, int row, float v) {
  switch (id) {
    case kSegIn: st_tagged(a.t + row, v, tg.t); break;
    case kSegQkvo: st_tagged(a.y + row, v, tg.y); break;
    case kSegIf: {
      const float t = __fadd_rn(v, a.L.b_if[row]);
      st_tagged_f32(a.g + row, __fmul_rn(a.cap, static_cast<float>(tanh(static_cast<double>(__fdiv_rn(t, a.cap))))),
                    tg.y);
      break;
    }
    case kSegOut: st_tagged(a.wo + row, v, tg.wo); break;
    case kSegDown: st_tagged(a.dn + row, v, tg.dn); break;
    case kSegHead:
      if (a.decoder) {
        a.logits[row] = v;
        st_tagged_f32(a.lg + row, v, tg.lg);
      } else {
        a.patch_out[row] = __float2bfloat16_rn(v);
      }
      break;
    case kSegBnd:
      *a.boundary_logit = v;
      if (a.fused) st_tagged_f32(a.bnd, v, tg.bnd);  // read by this launch's decoder part
      break;
    default: break;
  }
}

// A K = 2048 segment whose first chunk is number `off` of its phase: warp w takes the phase's chunks w,
// w + 8, ... whole (4 rows at once), so that the striding the ring waits rely on runs across the segments
// of a phase (see persist.cuh, acquire); returns the next chunk.
__device__ uint32_t gemv_seg(const Args& a, const Tags& tg, Smem& s, const Seg& sg, int id, uint32_t j0, const float (&xr)[64],
                             int off = 0) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nch = sg.chunks();
  for (int ch = (warp - off % kConsumerWarps + kConsumerWarps) % kConsumerWarps; ch < nch; ch += kConsumerWarps) {
    const uint8_t* slot = acquire(s.r, j0 + ch);
    if (slot == nullptr) break;
    float v[4];
    dot4x2048(slot, xr, v);
    release(s.r, j0 + ch, 1);
    if (sg.pair_off > 0) {  // gate (even chunks) and up (odd chunks) rows of the same indices
      const int rl = (ch / 2) * 4 + lane;
      if (lane < 4 && sg.r0 + rl < sg.r1) ((ch & 1) ? s.ubuf : s.gbuf)[rl] = lane_row(v);
    } else {
      const int row = sg.r0 + ch * sg.rpc + lane;
      if (lane < sg.rpc && lane < 4 && row < sg.r1) store_row(a, tg, id, row, lane_row(v));
    }
  }
  return j0 + nch;
}

// The down segment: K = 2816, 2 rows per chunk, x in s.vec; warp w takes the chunks w, w + 8, ...
__device__ uint32_t gemv_down(const Args& a, const Tags& tg, Smem& s, const Seg& sg, uint32_t j0) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nch = sg.chunks();
  for (int ch = warp; ch < nch; ch += kConsumerWarps) {
    const uint8_t* slot = acquire(s.r, j0 + ch);
    if (slot == nullptr) break;
    float acc[2][2] = {{0.0f, 0.0f}, {0.0f, 0.0f}};
#pragma unroll
    for (int i = 0; i < kFfn / 256; ++i) {
      float x[8];
      unpack8(*reinterpret_cast<const uint4*>(&s.vec[lane * 8 + 256 * i]), x);
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        float w[8];
        unpack8(*reinterpret_cast<const uint4*>(slot + r * kFfn * 2 + (lane * 8 + 256 * i) * 2), w);
#pragma unroll
        for (int jj = 0; jj < 8; ++jj) acc[r][jj & 1] = fmaf(w[jj], x[jj], acc[r][jj & 1]);
      }
    }
    release(s.r, j0 + ch, 1);
    float v[2] = {acc[0][0] + acc[0][1], acc[1][0] + acc[1][1]};
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
#pragma unroll
      for (int r = 0; r < 2; ++r) v[r] += __shfl_xor_sync(kFull, v[r], o);
    const int row = sg.r0 + ch * 2 + lane;
    if (lane < 2 && row < sg.r1) st_tagged(a.dn + row, lane == 0 ? v[0] : v[1], tg.dn);
  }
  return j0 + nch;
}

// ---- the mLSTM step of one unit (head hd, value columns c0 .. c0 + 15) -------------------------------------
// Thread t owns the column pair cp = t % 8 (columns c0 + 2 cp, + 1) and the rows t / 8 + 32 i (i < 16) of
// the tile, and the two n rows 2 t, 2 t + 1.
// q, k, v and the gates come from the tagged hand-off of the qkvo phase; false when the step stops (every
// consumer still reaches the CTA barriers inside).
__device__ bool mlstm_unit(const Args& a, const Tags& tg, unsigned* sy, Smem& s, int hd, int c0) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const Layer& L = a.L;
  const uint32_t* q = a.y + hd * kDh;
  const uint32_t* k = a.y + kD + hd * kDh;
  const uint32_t* v = a.y + 2 * kD + hd * kDh + c0;
  const int r = 2 * tid, cp = tid % 8, rb = tid / 8;
  // the state first (it does not wait for the hand-off)
  float* cbase = L.c + static_cast<size_t>(hd) * kDh * kDh + c0 + 2 * cp;
  constexpr int kRowsPerThread = kDh / 32;
  float2 cv[kRowsPerThread];  // all 16 loads in flight before the first store
#pragma unroll
  for (int i = 0; i < kRowsPerThread; ++i) cv[i] = *reinterpret_cast<const float2*>(cbase + static_cast<size_t>(rb + 32 * i) * kDh);
  const float2 n2 = *reinterpret_cast<const float2*>(L.n_cur + hd * kDh + r);
  const float m_old = L.m_cur[hd];
  // every hand-off load of this thread in flight at once, then the tag checks: the gates, its q and k pair,
  // its v pair
  const uint64_t gi = ld_relaxed8(a.g + hd), gf = ld_relaxed8(a.g + kNH + hd);
  const uint32_t wk0 = ld_relaxed4(k + r), wk1 = ld_relaxed4(k + r + 1), wq0 = ld_relaxed4(q + r),
                 wq1 = ld_relaxed4(q + r + 1), wv0 = ld_relaxed4(v + 2 * cp), wv1 = ld_relaxed4(v + 2 * cp + 1);
  float iv, fv, k0, k1, q0, q1, va, vb;
  bool ok = take_tagged_f32(gi, a.g + hd, tg.y, iv, sy);
  ok &= take_tagged_f32(gf, a.g + kNH + hd, tg.y, fv, sy);
  ok &= take_tagged1(wk0, k + r, tg.y, k0, sy);
  ok &= take_tagged1(wk1, k + r + 1, tg.y, k1, sy);
  ok &= take_tagged1(wq0, q + r, tg.y, q0, sy);
  ok &= take_tagged1(wq1, q + r + 1, tg.y, q1, sy);
  ok &= take_tagged1(wv0, v + 2 * cp, tg.y, va, sy);
  ok &= take_tagged1(wv1, v + 2 * cp + 1, tg.y, vb, sy);
  // gates (every thread; the scan kernel's gate_chunk for one position)
  const float ex = static_cast<float>(exp(-static_cast<double>(fv)));
  const float sig = __fdiv_rn(1.0f, __fadd_rn(1.0f, ex));
  const float fl = static_cast<float>(log(static_cast<double>(sig)));
  const float sum = __fadd_rn(fl, m_old);
  const float mn = fmaxf(sum, iv);
  const float g_mx = round_bf16(static_cast<float>(exp(-static_cast<double>(mn))));
  const float fa = round_bf16(static_cast<float>(exp(static_cast<double>(__fsub_rn(sum, mn)))));
  const float ia = round_bf16(static_cast<float>(exp(static_cast<double>(__fsub_rn(iv, mn)))));
  const float qsc = round_bf16(a.qk_scale);
  // n rows 2 t, 2 t + 1 and their part of q . n
  float qn = 0.0f;
  {
    const float n0 = fmaf(fa, n2.x, round_bf16(__fmul_rn(ia, k0)));
    const float n1 = fmaf(fa, n2.y, round_bf16(__fmul_rn(ia, k1)));
    if (c0 == 0) *reinterpret_cast<float2*>(L.n_next + hd * kDh + r) = make_float2(n0, n1);
    const float qs0 = round_bf16(__fmul_rn(q0, qsc)), qs1 = round_bf16(__fmul_rn(q1, qsc));
    s.kf[r] = k0;
    s.kf[r + 1] = k1;
    s.qsv[r] = qs0;
    s.qsv[r + 1] = qs1;
    const float p0 = round_bf16(__fmul_rn(qs0, round_bf16(n0)));
    const float p1 = round_bf16(__fmul_rn(qs1, round_bf16(n1)));
    qn = p0 + p1;
  }
  qn = consumer_sum(qn, s.r.red[1]);  // also makes s.kf, s.qsv visible
  if (c0 == 0 && tid == 0) L.m_next[hd] = mn;
  // the C tile
  float ha = 0.0f, hb = 0.0f;
#pragma unroll
  for (int i = 0; i < kRowsPerThread; ++i) {
    const int r = rb + 32 * i;
    const float kr = s.kf[r], qs = s.qsv[r];
    const float ua = round_bf16(__fmul_rn(ia, round_bf16(__fmul_rn(kr, va))));
    const float ub = round_bf16(__fmul_rn(ia, round_bf16(__fmul_rn(kr, vb))));
    cv[i].x = fmaf(fa, cv[i].x, ua);
    cv[i].y = fmaf(fa, cv[i].y, ub);
    ha += round_bf16(__fmul_rn(qs, round_bf16(cv[i].x)));
    hb += round_bf16(__fmul_rn(qs, round_bf16(cv[i].y)));
  }
#pragma unroll
  for (int i = 0; i < kRowsPerThread; ++i) *reinterpret_cast<float2*>(cbase + static_cast<size_t>(rb + 32 * i) * kDh) = cv[i];
  // column sums: the 4 lanes of this warp with the same cp (xor 8, 16), then the warps in order
  ha += __shfl_xor_sync(kFull, ha, 8);
  hb += __shfl_xor_sync(kFull, hb, 8);
  ha += __shfl_xor_sync(kFull, ha, 16);
  hb += __shfl_xor_sync(kFull, hb, 16);
  if (lane < 8) {
    s.part[warp][2 * lane] = ha;
    s.part[warp][2 * lane + 1] = hb;
  }
  consumer_sync();
  if (tid < kCols) {
    float hs = 0.0f;
#pragma unroll
    for (int w = 0; w < kConsumerWarps; ++w) hs += s.part[w][tid];
    const float den = __fadd_rn(fmaxf(fabsf(qn), g_mx), a.mlstm_eps);
    st_tagged(a.hm + hd * kDh + c0 + tid, __fdiv_rn(hs, den), tg.hm);
  }
  consumer_sync();  // s.part and s.r.red are reused by the next unit
  return ok;
}

// ---- the consumers ----------------------------------------------------------------------------------------
// Hand-offs between the phases go through tagged words (persist.cuh) behind grid barriers without fence: the
// ordered barrier's release fence waited for the SM's bulk copies in flight.
// j: the ring chunk counter, epoch: the grid barriers passed (both carried from a fused launch's encoder part
// into its decoder part).
__device__ void consumers(const Args& a, Smem& s, const Plan& pl, int c, int G, const Pre& pre, const Tags& tg,
                          uint32_t& j, unsigned& epoch) {
  const int tid = threadIdx.x, e = tid * 8;
  float xr[64];
  auto stop = [&]() { return consumers_stop(s.r, a.sync); };
  auto signal = [&]() { return grid_sync(s.r, a.sync, epoch, false); };
  // decoder: t = W_in e
  if (a.decoder) {
    *reinterpret_cast<uint4*>(&s.vec[e]) = pre.x0;
    consumer_sync();
    load_lane_x(s.vec, xr);
    j = gemv_seg(a, tg, s, pl.seg[kSegIn], kSegIn, j, xr);
    if (stop() || !signal()) return;
  }
  // x = rmsnorm(h) * norm1; y = W_qkvo x; g = soft-capped gates
  {
    float h[8];
    const bool ok = layer_input(a, tg, a.sync, h, pre);
    norm_into_vec(s, h, pre.n1, a.eps);
    if (consumers_stop_if(s.r, a.sync, !ok)) return;  // also the CTA barrier after s.vec
    load_lane_x(s.vec, xr);
    j = gemv_seg(a, tg, s, pl.seg[kSegQkvo], kSegQkvo, j, xr);
    j = gemv_seg(a, tg, s, pl.seg[kSegIf], kSegIf, j, xr, pl.seg[kSegQkvo].chunks());
    if (stop() || !signal()) return;
  }
  // the mLSTM step
  {
    bool ok = true;
    for (int u = c; u < kUnits; u += G) ok &= mlstm_unit(a, tg, a.sync, s, u / (kDh / kCols), (u % (kDh / kCols)) * kCols);
    if (consumers_stop_if(s.r, a.sync, !ok) || !signal()) return;
  }
  // z = bf16(bf16(sigmoid(o)) * bf16(rmsnorm_head(hm) * mh_norm)); wo = W_out z
  {
    const int hd = e / kDh;  // 64 threads (2 warps) per head
    const uint4 h0 = ld_relaxed16(a.hm + e), h1 = ld_relaxed16(a.hm + e + 4);
    const uint4 o0 = ld_relaxed16(a.y + 3 * kD + e), o1 = ld_relaxed16(a.y + 3 * kD + e + 4);
    float f[8], ov[8];
    bool ok = take_tagged8(h0, h1, a.hm + e, tg.hm, f, a.sync);
    ok &= take_tagged8(o0, o1, a.y + 3 * kD + e, tg.y, ov, a.sync);
    float ss = 0.0f;
#pragma unroll
    for (int jj = 0; jj < 8; ++jj) ss = fmaf(f[jj], f[jj], ss);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(kFull, ss, o);
    if ((tid & 31) == 0) s.head_red[hd][(tid >> 5) & 1] = ss;
    consumer_sync();
    const float inv = inv_rms(s.head_red[hd][0] + s.head_red[hd][1], kDh, a.eps);
    float wv[8], z[8];
    unpack8(pre.mh, wv);
#pragma unroll
    for (int jj = 0; jj < 8; ++jj)
      z[jj] = __fmul_rn(round_bf16(sigmoid_d(ov[jj])), round_bf16(__fmul_rn(__fmul_rn(f[jj], inv), wv[jj])));
    *reinterpret_cast<uint4*>(&s.vec[e]) = pack8(z);
    if (consumers_stop_if(s.r, a.sync, !ok)) return;  // also the CTA barrier after s.vec
    load_lane_x(s.vec, xr);
    j = gemv_seg(a, tg, s, pl.seg[kSegOut], kSegOut, j, xr);
    if (stop() || !signal()) return;
  }
  // x2 = rmsnorm(h2) * norm2; a = silu(W_gate x2) * (W_up x2)
  {
    float h2[8];
    const bool ok = layer_h2(a, tg, a.sync, h2, pre);
    norm_into_vec(s, h2, pre.n2, a.eps);
    if (consumers_stop_if(s.r, a.sync, !ok)) return;
    load_lane_x(s.vec, xr);
    const Seg& sg = pl.seg[kSegGu];
    j = gemv_seg(a, tg, s, sg, kSegGu, j, xr);
    if (stop()) return;
    for (int rl = tid; rl < sg.r1 - sg.r0; rl += kConsumers) {
      const float gv = round_bf16(s.gbuf[rl]), up = round_bf16(s.ubuf[rl]);
      const float sl = round_bf16(static_cast<float>(gv / (1.0 + exp(-static_cast<double>(gv)))));
      st_tagged(a.a + sg.r0 + rl, __fmul_rn(sl, up), tg.a);
    }
    if (!signal()) return;
  }
  // dn = W_down a
  {
    constexpr int kGroups = (kFfn / 8 + kConsumers - 1) / kConsumers;  // 8-value groups per thread (2)
    uint4 ua[kGroups][2];  // all loads in flight, then the tag checks
#pragma unroll
    for (int q = 0; q < kGroups; ++q) {
      const int i = tid + q * kConsumers;
      if (i < kFfn / 8) {
        ua[q][0] = ld_relaxed16(a.a + i * 8);
        ua[q][1] = ld_relaxed16(a.a + i * 8 + 4);
      }
    }
    bool ok = true;
#pragma unroll
    for (int q = 0; q < kGroups; ++q) {
      const int i = tid + q * kConsumers;
      if (i < kFfn / 8) {
        float f[8];
        ok &= take_tagged8(ua[q][0], ua[q][1], a.a + i * 8, tg.a, f, a.sync);
        *reinterpret_cast<uint4*>(&s.vec[i * 8]) = pack8(f);
      }
    }
    if (consumers_stop_if(s.r, a.sync, !ok)) return;
    j = gemv_down(a, tg, s, pl.seg[kSegDown], j);
    if (stop() || !signal()) return;
  }
  // the layer output, its norm, and the head (patch + boundary, or the LM head)
  {
    float h2[8], d[8], out[8];
    const uint4 d0 = ld_relaxed16(a.dn + e), d1 = ld_relaxed16(a.dn + e + 4);
    bool ok = layer_h2(a, tg, a.sync, h2, pre);
    ok &= take_tagged8(d0, d1, a.dn + e, tg.dn, d, a.sync);
#pragma unroll
    for (int jj = 0; jj < 8; ++jj) out[jj] = round_bf16(__fadd_rn(h2[jj], d[jj]));
    norm_into_vec(s, out, pre.on, a.eps);
    if (consumers_stop_if(s.r, a.sync, !ok)) return;
    if (!a.decoder && c == 0) *reinterpret_cast<uint4*>(a.e_out + e) = *reinterpret_cast<const uint4*>(&s.vec[e]);
    load_lane_x(s.vec, xr);
    j = gemv_seg(a, tg, s, pl.seg[kSegHead], kSegHead, j, xr);
    if (!a.decoder) j = gemv_seg(a, tg, s, pl.seg[kSegBnd], kSegBnd, j, xr, pl.seg[kSegHead].chunks());
    if (stop()) return;
  }
  if (!a.decoder) return;
  if (!signal()) return;
  // decoder: out = [argmax(logits) (torch order: NaN largest, lowest index on ties), boundary flag]
  if (c != 0) return;
  float best = -INFINITY;
  int idx = 0x7fffffff;
  auto better = [](float x, int ix, float y, int iy) {
    const bool nx = isnan(x), ny = isnan(y);
    if (nx || ny) return nx && (!ny || ix < iy);
    return x > y || (x == y && ix < iy);
  };
  constexpr int kPer = (kVocab + kConsumers - 1) / kConsumers;  // logits per thread (2)
  uint64_t wl[kPer];
#pragma unroll
  for (int q = 0; q < kPer; ++q)
    if (tid + q * kConsumers < kVocab) wl[q] = ld_relaxed8(a.lg + tid + q * kConsumers);
  bool lok = true;
#pragma unroll
  for (int q = 0; q < kPer; ++q) {
    const int i = tid + q * kConsumers;
    if (i >= kVocab) continue;
    float x;
    lok &= take_tagged_f32(wl[q], a.lg + i, tg.lg, x, a.sync);
    if (better(x, i, best, idx)) {
      best = x;
      idx = i;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ob = __shfl_xor_sync(kFull, best, o);
    const int oi = __shfl_xor_sync(kFull, idx, o);
    if (better(ob, oi, best, idx)) {
      best = ob;
      idx = oi;
    }
  }
  if ((tid & 31) == 0) {
    s.part[tid >> 5][0] = best;
    s.part[tid >> 5][1] = __int_as_float(idx);
  }
  const bool bad = named_barrier_or(1, kConsumers, !lok);  // a failed wait leaves out alone
  if (tid == 0 && !bad) {
    for (int w = 1; w < kConsumerWarps; ++w) {
      const float ob = s.part[w][0];
      const int oi = __float_as_int(s.part[w][1]);
      if (better(ob, oi, best, idx)) {
        best = ob;
        idx = oi;
      }
    }
    float bl = *a.boundary_logit;
    if (a.fused && !take_tagged_f32(ld_relaxed8(a.bnd), a.bnd, tg.bnd, bl, a.sync)) return;
    a.out[0] = idx;
    a.out[1] = sigmoid_d(bl) >= 0.5f ? 1 : 0;
  }
}

__global__ void __launch_bounds__(kThreads, 1) loc_step_kernel(Args a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  Smem& s = *reinterpret_cast<Smem*>(smem_raw);
  const int c = blockIdx.x, G = gridDim.x;
  long long byte = 0;
  bool valid = true;
  if (!a.decoder) {
    byte = *a.byte;
    valid = byte >= 0 && byte < kVocab;  // the same answer in every CTA
  }
  // the consumers' loads that no phase waits for go out while the first producer thread builds the plan
  const unsigned seq = *reinterpret_cast<volatile unsigned*>(a.sync + 8);  // this launch's number (tags)
  Pre pre{};
  if (threadIdx.x < kConsumers && valid) {
    pre.load(a, byte);
  }
  if (threadIdx.x == kConsumers) {
    s.plan.init(a, c, G);
    if (a.fused) {  // the decoder part: the same arguments with its layer
      s.part1 = a;
      s.part1.L = a.L2;
      s.part1.decoder = 1;
      s.plan1.init(s.part1, c, G);
    }
    ring_init(s.r);
  }
  __syncthreads();
  const Plan& pl = s.plan;
  if (threadIdx.x >= kConsumers) {
    if ((threadIdx.x & 31) == 0) {
      const Stream2 src{pl, a.fused ? &s.plan1 : nullptr};
      produce<kProducers>(s.r, src, valid ? src.total() : 0, (threadIdx.x - kConsumers) / 32);
    }
    return;
  }
  if (!valid) {  // host checks keep the byte in range; never index with a bad one
    if (c == 0) {
      const uint4 nan4 = make_uint4(0x7fc07fc0u, 0x7fc07fc0u, 0x7fc07fc0u, 0x7fc07fc0u);
      *reinterpret_cast<uint4*>(a.e_out + threadIdx.x * 8) = nan4;
      *reinterpret_cast<uint4*>(a.patch_out + threadIdx.x * 8) = nan4;
      if (threadIdx.x == 0) *a.boundary_logit = __int_as_float(0x7fc00000);
    }
    return;
  }
  uint32_t j = 0;
  unsigned epoch = 0;
  consumers(a, s, pl, c, G, pre, Tags(seq, 0), j, epoch);
  const bool stopped = named_barrier_or(1, kConsumers, s.r.abort != 0);  // one answer for every consumer
  if (a.fused && !stopped) {
    // the decoder part, in the same ring and barrier sequence; its input e is this CTA's s.vec (the encoder
    // part's normalised output, also in e_out)
    Pre pd{};
    pd.load(s.part1, 0);
    pd.x0 = *reinterpret_cast<const uint4*>(&s.vec[threadIdx.x * 8]);
    consumers(s.part1, s, s.plan1, c, G, pd, Tags(seq, 8), j, epoch);
  }
  // CTA 0 finishes after every CTA has read the number (they read it at their start)
  if (c == 0 && threadIdx.x == 0) *reinterpret_cast<volatile unsigned*>(a.sync + 8) = seq + 1;
}

constexpr size_t kWsT = 0;  // tagged hand-offs: 4 bytes per bf16 value, 8 per fp32 value
constexpr size_t kWsY = kWsT + kD * 4;
constexpr size_t kWsG = kWsY + 4 * kD * 4;
constexpr size_t kWsHm = kWsG + 256;
constexpr size_t kWsWo = kWsHm + kD * 4;
constexpr size_t kWsA = kWsWo + kD * 4;
constexpr size_t kWsDn = kWsA + kFfn * 4;
constexpr size_t kWsLg = kWsDn + kD * 4;
constexpr size_t kWsSync = kWsLg + kVocab * 8;
constexpr size_t kWsBytes = kWsSync + 256;

int launch_loc(Args& a, void* workspace, size_t workspace_bytes, cudaStream_t s) {
  if (workspace == nullptr || workspace_bytes < kWsBytes)
    return fail(BP_ERR_INVALID_ARGUMENT, "workspace NULL or too small (%zu < %zu bytes)", workspace_bytes, kWsBytes);
  if ((reinterpret_cast<uintptr_t>(workspace) & 15u) != 0) return fail(BP_ERR_MISALIGNED, "workspace must be 16-byte aligned");
  char* ws = static_cast<char*>(workspace);
  a.t = reinterpret_cast<uint32_t*>(ws + kWsT);
  a.y = reinterpret_cast<uint32_t*>(ws + kWsY);
  a.g = reinterpret_cast<uint64_t*>(ws + kWsG);
  a.hm = reinterpret_cast<uint32_t*>(ws + kWsHm);
  a.wo = reinterpret_cast<uint32_t*>(ws + kWsWo);
  a.a = reinterpret_cast<uint32_t*>(ws + kWsA);
  a.dn = reinterpret_cast<uint32_t*>(ws + kWsDn);
  a.lg = reinterpret_cast<uint64_t*>(ws + kWsLg);
  a.sync = reinterpret_cast<unsigned*>(ws + kWsSync);
  a.bnd = reinterpret_cast<uint64_t*>(ws + kWsSync + 64);  // kept (tagged), not cleared per launch
  a.qk_scale = 1.0f / sqrtf(static_cast<float>(kDh));
  int st = require_sm100();
  if (st != BP_OK) return st;
  const int sms = tc_sm_count();
  if ((kFfn + sms - 1) / sms > kMaxGuRows || sms < 2 * kNH) return fail(BP_ERR_UNSUPPORTED, "loc_step needs at least 44 SMs");
  const size_t smem = sizeof(Smem);
  cudaError_t e = cudaFuncSetAttribute(loc_step_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return fail(BP_ERR_CUDA, "loc_step smem attribute: %s", cudaGetErrorString(e));
  int per_sm = 0;
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, loc_step_kernel, kThreads, smem);
  if (e != cudaSuccess || per_sm < 1) return fail(BP_ERR_CUDA, "loc_step does not fit on an SM");
  e = cudaMemsetAsync(a.sync, 0, 16, s);  // arrival counter, abort word (the launch number stays)
  if (e != cudaSuccess) return fail(BP_ERR_CUDA, "loc_step sync reset: %s", cudaGetErrorString(e));
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
  e = cudaLaunchKernelEx(&cfg, loc_step_kernel, a);
  if (e != cudaSuccess) return fail(BP_ERR_CUDA, "loc_step launch: %s", cudaGetErrorString(e));
  return check_launch("loc_step");
}

bool a16(const void* p) { return p != nullptr && (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int fill_layer(const bp_loc_layer* l, Layer& L) {
  if (l == nullptr) return fail(BP_ERR_INVALID_ARGUMENT, "layer is NULL");
  const void* ptrs[] = {l->norm1, l->w_qkvo, l->w_if, l->b_if, l->mh_norm, l->w_out, l->norm2, l->w_gu, l->w_down,
                        l->c, l->n_cur, l->m_cur, l->n_next, l->m_next};
  for (const void* p : ptrs)
    if (!a16(p)) return fail(BP_ERR_MISALIGNED, "a layer pointer is NULL or not 16-byte aligned");
  if (l->n_cur == l->n_next || l->m_cur == l->m_next)
    return fail(BP_ERR_INVALID_ARGUMENT, "n / m must go to other buffers than they come from");
  L = Layer{static_cast<const __nv_bfloat16*>(l->norm1), static_cast<const __nv_bfloat16*>(l->w_qkvo),
            static_cast<const __nv_bfloat16*>(l->w_if), l->b_if, static_cast<const __nv_bfloat16*>(l->mh_norm),
            static_cast<const __nv_bfloat16*>(l->w_out), static_cast<const __nv_bfloat16*>(l->norm2),
            static_cast<const __nv_bfloat16*>(l->w_gu), static_cast<const __nv_bfloat16*>(l->w_down), l->c,
            l->n_cur, l->m_cur, l->n_next, l->m_next};
  return BP_OK;
}

}  // namespace

BP_DEFINE_DEVICE_ERROR_READER(read_device_errors_loc)

}  // namespace bp

extern "C" size_t bp_loc_step_workspace_bytes(void) { return bp::kWsBytes; }

extern "C" int bp_loc_enc_step(const bp_loc_layer* layer, const void* embed, const int64_t* byte, const void* enc_norm,
                               const void* w_patch, const void* w_boundary, void* e_out, void* patch_out,
                               float* boundary_logit, float eps, float gate_cap, float mlstm_eps, void* workspace,
                               size_t workspace_bytes, void* stream) {
  using namespace bp;
  clear_error();
  Args a{};
  int st = fill_layer(layer, a.L);
  if (st != BP_OK) return st;
  if (!a16(embed) || byte == nullptr || !a16(enc_norm) || !a16(w_patch) || !a16(w_boundary) || !a16(e_out) ||
      !a16(patch_out) || boundary_logit == nullptr)
    return fail(BP_ERR_MISALIGNED, "a pointer is NULL or not 16-byte aligned");
  a.decoder = 0;
  a.embed = static_cast<const __nv_bfloat16*>(embed);
  a.byte = reinterpret_cast<const long long*>(byte);
  a.enc_norm = static_cast<const __nv_bfloat16*>(enc_norm);
  a.w_patch = static_cast<const __nv_bfloat16*>(w_patch);
  a.w_boundary = static_cast<const __nv_bfloat16*>(w_boundary);
  a.e_out = static_cast<__nv_bfloat16*>(e_out);
  a.patch_out = static_cast<__nv_bfloat16*>(patch_out);
  a.boundary_logit = boundary_logit;
  a.eps = eps;
  a.cap = gate_cap;
  a.mlstm_eps = mlstm_eps;
  return launch_loc(a, workspace, workspace_bytes, static_cast<cudaStream_t>(stream));
}

extern "C" int bp_loc_dec_step(const bp_loc_layer* layer, const void* e_in, const void* value, const void* w_in,
                               const void* final_norm, const void* lm_head, const float* boundary_logit, float* logits,
                               int64_t* out, float eps, float gate_cap, float mlstm_eps, void* workspace,
                               size_t workspace_bytes, void* stream) {
  using namespace bp;
  clear_error();
  Args a{};
  int st = fill_layer(layer, a.L);
  if (st != BP_OK) return st;
  if (!a16(e_in) || !a16(value) || !a16(w_in) || !a16(final_norm) || !a16(lm_head) || boundary_logit == nullptr ||
      logits == nullptr || out == nullptr)
    return fail(BP_ERR_MISALIGNED, "a pointer is NULL or not 16-byte aligned");
  a.decoder = 1;
  a.e_in = static_cast<const __nv_bfloat16*>(e_in);
  a.value = static_cast<const __nv_bfloat16*>(value);
  a.w_in = static_cast<const __nv_bfloat16*>(w_in);
  a.final_norm = static_cast<const __nv_bfloat16*>(final_norm);
  a.lm_head = static_cast<const __nv_bfloat16*>(lm_head);
  a.boundary_logit = const_cast<float*>(boundary_logit);
  a.logits = logits;
  a.out = reinterpret_cast<long long*>(out);
  a.eps = eps;
  a.cap = gate_cap;
  a.mlstm_eps = mlstm_eps;
  return launch_loc(a, workspace, workspace_bytes, static_cast<cudaStream_t>(stream));
}

extern "C" int bp_loc_encdec_step(const bp_loc_layer* enc_layer, const bp_loc_layer* dec_layer, const void* embed,
                                  const int64_t* byte, const void* enc_norm, const void* w_patch,
                                  const void* w_boundary, void* e_out, void* patch_out, float* boundary_logit,
                                  const void* value, const void* w_in, const void* final_norm, const void* lm_head,
                                  float* logits, int64_t* out, float eps, float gate_cap, float mlstm_eps,
                                  void* workspace, size_t workspace_bytes, void* stream) {
  using namespace bp;
  clear_error();
  Args a{};
  int st = fill_layer(enc_layer, a.L);
  if (st != BP_OK) return st;
  st = fill_layer(dec_layer, a.L2);
  if (st != BP_OK) return st;
  if (a.L.c == a.L2.c || a.L.n_next == a.L2.n_next || a.L.m_next == a.L2.m_next)
    return fail(BP_ERR_INVALID_ARGUMENT, "the encoder and decoder layers must have their own state");
  if (!a16(embed) || byte == nullptr || !a16(enc_norm) || !a16(w_patch) || !a16(w_boundary) || !a16(e_out) ||
      !a16(patch_out) || boundary_logit == nullptr || !a16(value) || !a16(w_in) || !a16(final_norm) ||
      !a16(lm_head) || logits == nullptr || out == nullptr)
    return fail(BP_ERR_MISALIGNED, "a pointer is NULL or not 16-byte aligned");
  a.decoder = 0;
  a.fused = 1;
  a.embed = static_cast<const __nv_bfloat16*>(embed);
  a.byte = reinterpret_cast<const long long*>(byte);
  a.enc_norm = static_cast<const __nv_bfloat16*>(enc_norm);
  a.w_patch = static_cast<const __nv_bfloat16*>(w_patch);
  a.w_boundary = static_cast<const __nv_bfloat16*>(w_boundary);
  a.e_out = static_cast<__nv_bfloat16*>(e_out);
  a.patch_out = static_cast<__nv_bfloat16*>(patch_out);
  a.boundary_logit = boundary_logit;
  a.e_in = static_cast<const __nv_bfloat16*>(e_out);  // the decoder part takes e from shared memory
  a.value = static_cast<const __nv_bfloat16*>(value);
  a.w_in = static_cast<const __nv_bfloat16*>(w_in);
  a.final_norm = static_cast<const __nv_bfloat16*>(final_norm);
  a.lm_head = static_cast<const __nv_bfloat16*>(lm_head);
  a.logits = logits;
  a.out = reinterpret_cast<long long*>(out);
  a.eps = eps;
  a.cap = gate_cap;
  a.mlstm_eps = mlstm_eps;
  return launch_loc(a, workspace, workspace_bytes, static_cast<cudaStream_t>(stream));
}
