// Fused mLSTM recurrence over T positions with the (C, n, m) state kept on chip, plus the draft
// acceptance kernel.
//
// Reference: byteprof/optim/mlstm_multistep.py:20-146 (_gates, multistep_fw_kernel,
// lazy_commit_kernel, accept_kernel) and the library step it restates (mlstm_kernels 2.0.6
// recurrent_step_fw_kernel, called at byteprof/optim/draft_core.py:114-141).
//
// Per position t and head (reference math, mlstm_multistep.py:20-30, 64-85):
//   f_log = log(sigmoid(f_t)),  m_t = max(f_log + m_{t-1}, i_t)
//   f_act = exp(f_log + m_{t-1} - m_t),  i_act = exp(i_t - m_t),  max_val = exp(-m_t)
//   C_t = f_act * C_{t-1} + i_act * (k_t v_t^T),  n_t = f_act * n_{t-1} + i_act * k_t
//   h_t = (q_t * qk_scale)^T C_t / (max(|(q_t * qk_scale)^T n_t|, max_val) + eps)
// With bf16 inputs the reference rounds to bf16: f_act, i_act, max_val (.to(DTYPE)), k*v and
// i_act*(k*v) (bf16 x bf16 stays bf16 under Triton's promotion rules), q*qk_scale (the scalar is
// cast to bf16 first), C and n before the output dot products and each product q*C, q*n. This
// kernel applies the same roundings. It accumulates the two dot products in fp32 (the reference
// reduces the bf16 products in bf16, in an order that depends on its register layout).
// The gate values are evaluated in double precision and rounded to fp32 at each point where the
// reference holds an fp32 value, so the bf16 gate values are the correctly rounded ones.
//
// B200 design: grid (DV / 16, NH); each CTA owns 16 value columns of one head and keeps that
// [DQ x 16] fp32 slice of C in registers for all T positions (no per-position HBM round trip of the
// 4 MiB state). TPC threads share one column (RPT rows each, in 8-row chunks so that q and k are
// read from shared memory with 16-byte loads). One extra producer warp per CTA
//   - prefetches q, k, v of position t + 7 with cp.async into an 8-deep shared-memory ring,
//   - evaluates the gate recurrence 32 positions at a time (double buffered),
//   - updates n and the q.n denominator, and finishes h_t one position later.
// One __syncthreads per position. (head, column-block) CTAs are independent: no inter-CTA waits.
#include "bp_common.cuh"

namespace bp {
namespace {

constexpr int kBV = 16;    // value columns per CTA
constexpr int kDepth = 8;  // shared-memory ring depth (positions)
constexpr int kGC = 32;    // gate chunk (positions)

struct ScanArgs {
  const float* c_in;
  const float* n_in;
  const float* m_in;
  const void* q;
  const void* k;
  const void* v;
  const void* ig;
  const void* fg;
  void* h;
  float* c_out;
  float* n_out;
  float* m_out;
  float* n_save;
  float* m_save;
  const int64_t* steps_dev;
  int T, NH, DV;
  long long str_qk, str_v, str_if, str_h;
  int gate_f32;
  int stage_c;  // C moves through shared memory with 16-byte copies (c_in and c_out 16-byte aligned)
  float qk_scale, eps;
};

// The CTA's [DQ x 16] fp32 block of C moves between global memory and the compute threads' registers
// through shared memory, so that every warp access covers whole 64-byte rows (with per-thread scalar
// accesses a warp touches 16 rows x 8 bytes, four times the L2 requests for the same bytes). Word of
// (row r, column c): row r sits in physical row r ^ ((r >> 5) & 1), its 16-byte chunk c / 4 in slot
// (c / 4) ^ ((r >> 3) & 3). A compute thread's access to rows 8l + e (l = 0..15, e fixed) then spreads
// the 32 lanes over 16 banks (two lanes per bank, the minimum for the warp's two columns), while 8
// consecutive rows stay one contiguous 512-byte run for the chunk copies.
__device__ __forceinline__ int stage_word(int r, int c) {
  return (r ^ ((r >> 5) & 1)) * kBV + (((c >> 2) ^ ((r >> 3) & 3)) << 2) + (c & 3);
}

__device__ __forceinline__ void compute_sync(int nthreads) { asm volatile("bar.sync 1, %0;" ::"r"(nthreads) : "memory"); }

template <typename T>
__device__ __forceinline__ float to_f(T v);
template <>
__device__ __forceinline__ float to_f<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }

template <typename T>
__device__ __forceinline__ T from_f(float v);
template <>
__device__ __forceinline__ float from_f<float>(float v) { return v; }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }

// Rounds to the input dtype (the reference's `.to(DTYPE)`): bf16 rounds, fp32 is the identity.
template <typename T>
__device__ __forceinline__ float rnd(float v) {
  if constexpr (sizeof(T) == 2) return round_bf16(v);
  return v;
}

// Two adjacent elements of q or k from shared memory as floats (one 4- or 8-byte load).
template <typename T>
__device__ __forceinline__ void load_pair(const T* p, float& a, float& b) {
  if constexpr (sizeof(T) == 2) {
    const uint32_t w = *reinterpret_cast<const uint32_t*>(p);
    a = bf16lo(w);
    b = bf16hi(w);
  } else {
    const float2 v = *reinterpret_cast<const float2*>(p);
    a = v.x;
    b = v.y;
  }
}

// bf16 pair from two bf16-valued floats (exact), and back.
__device__ __forceinline__ __nv_bfloat162 pack2(float a, float b) { return __floats2bfloat162_rn(a, b); }
__device__ __forceinline__ void unpack2(__nv_bfloat162 v, float& a, float& b) {
  const float2 f = __bfloat1622float2(v);
  a = f.x;
  b = f.y;
}

// (o0, o1) = s * (a0, a1): with bf16 inputs one packed bf16 multiply (round to nearest), else fp32.
template <typename T>
__device__ __forceinline__ void mul_pair(float s, float a0, float a1, float& o0, float& o1) {
  if constexpr (sizeof(T) == 2) {
    unpack2(__hmul2(pack2(s, s), pack2(a0, a1)), o0, o1);
  } else {
    o0 = s * a0;
    o1 = s * a1;
  }
}

// (q0 * qsc) * c0 + (q1 * qsc) * c1 with the reference's bf16 roundings of q*qsc, c and each product
// (qsc is already bf16-valued in bf16 mode); the two products are added in fp32.
template <typename T>
__device__ __forceinline__ float dot_pair(float q0, float q1, float qsc, float c0, float c1) {
  if constexpr (sizeof(T) == 2) {
    const __nv_bfloat162 qs = __hmul2(pack2(q0, q1), pack2(qsc, qsc));
    float p0, p1;
    unpack2(__hmul2(qs, __floats2bfloat162_rn(c0, c1)), p0, p1);
    return p0 + p1;
  } else {
    return (q0 * qsc) * c0 + (q1 * qsc) * c1;
  }
}

template <int DQ, typename T>
struct ScanCfg {
  static constexpr int TPC = DQ >= 128 ? 16 : 8;  // threads per value column
  static constexpr int RPT = DQ / TPC;            // rows of C per thread
  static constexpr int CH = RPT / 8;              // 8-row chunks per thread
  static constexpr int NCOMP = kBV * TPC;         // compute threads
  static constexpr int NTHREADS = NCOMP + 32;     // + one producer warp
  static constexpr int RPL = DQ / 32;             // rows of n per producer lane: pairs 2*lane + 64*j + {0,1}
  static constexpr int STAGE = 2 * DQ + kBV;      // elements of q, k, v for one position
  static constexpr int CHUNKS16 = STAGE * static_cast<int>(sizeof(T)) / 16;
};

__device__ __forceinline__ float load_gate(const void* p, long long idx, int is_f32) {
  if (is_f32) return static_cast<const float*>(p)[idx];
  return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[idx]);
}

// Gate values of positions [32 j, 32 j + 32) of one head into slot (position & 63) of the gate
// buffers. `m_run` is the stabiliser after position 32 j - 1 on entry and after the last valid
// position of the chunk on exit (identical in every lane).
template <typename T>
__device__ __forceinline__ void gate_chunk(const ScanArgs& a, int head, int j, int n_steps, float& m_run, float* g_f, float* g_i,
                           float* g_mx) {
  const int lane = threadIdx.x & 31;
  const int s = j * kGC + lane;
  float fl = 0.0f, iv = 0.0f;
  if (s < n_steps) {
    const float fv = load_gate(a.fg, s * a.str_if + head, a.gate_f32);
    iv = load_gate(a.ig, s * a.str_if + head, a.gate_f32);
    // sigmoid(x) = 1 / (1 + exp(-x)) with fp32 intermediates, then log.
    const float e = static_cast<float>(exp(-static_cast<double>(fv)));
    const float d = __fadd_rn(1.0f, e);
    const float sig = __fdiv_rn(1.0f, d);
    fl = static_cast<float>(log(static_cast<double>(sig)));
  }
  // The stabiliser recurrence is sequential (each fp32 add rounds): every lane runs it, over the
  // chunk's valid positions only (`count` is the same in every lane).
  const int count = min(kGC, n_steps - j * kGC);
  float m_prev = m_run, my_m = 0.0f, my_a = 0.0f;
  for (int t = 0; t < count; ++t) {
    const float flt = __shfl_sync(0xffffffffu, fl, t);
    const float ivt = __shfl_sync(0xffffffffu, iv, t);
    const float sum = __fadd_rn(flt, m_prev);
    const float mn = fmaxf(sum, ivt);
    if (lane == t) {
      my_m = mn;
      my_a = __fsub_rn(sum, mn);
    }
    m_prev = mn;
  }
  m_run = m_prev;
  if (s < n_steps) {
    const int slot = s & 63;
    g_mx[slot] = rnd<T>(static_cast<float>(exp(-static_cast<double>(my_m))));
    g_f[slot] = rnd<T>(static_cast<float>(exp(static_cast<double>(my_a))));
    g_i[slot] = rnd<T>(static_cast<float>(exp(static_cast<double>(__fsub_rn(iv, my_m)))));
  }
}

template <int DQ, typename T>
__global__ void __launch_bounds__(ScanCfg<DQ, T>::NTHREADS) mlstm_scan_kernel(const ScanArgs a) {
  using Cfg = ScanCfg<DQ, T>;
  __shared__ __align__(16) T ring[kDepth][Cfg::STAGE];
  __shared__ float g_f[64], g_i[64], g_mx[64];
  __shared__ float hb[2][kBV];
  extern __shared__ __align__(16) float cst[];  // [DQ x 16] C staging (stage_word layout) when a.stage_c

  // Everything the scan reads (state, q, k, v, gates, the step count) may come from the kernels before it.
  // The next kernel launches when the scan exits, not earlier: an early launch_dependents let the next
  // weight stream start during the scan and made a local decode step 2-5 us slower (measured A/B), as its
  // loads queue beside the scan's latency-bound state reads.
  pdl_wait_prior_grids();

  const int head = blockIdx.y;
  const int c0 = blockIdx.x * kBV;
  const int tid = threadIdx.x;
  const bool producer = tid >= Cfg::NCOMP;
  const int lane = tid & 31;
  const bool want_h = a.h != nullptr;

  int n_steps = a.T;
  if (a.steps_dev != nullptr) {
    long long L = *a.steps_dev + 1;
    n_steps = static_cast<int>(L < 0 ? 0 : (L > a.T ? a.T : L));
  }

  const T* qg = static_cast<const T*>(a.q);
  const T* kg = static_cast<const T*>(a.k);
  const T* vg = static_cast<const T*>(a.v);

  // Producer: issue the copies of position s into ring slot s % kDepth (one commit group per call).
  auto issue = [&](int s) {
    if (s < n_steps) {
      T* dst = ring[s % kDepth];
      for (int c = lane; c < Cfg::CHUNKS16; c += 32) {
        constexpr int per_row = DQ * static_cast<int>(sizeof(T)) / 16;  // 16-byte chunks of q (or k)
        const char* src;
        if (c < per_row)
          src = reinterpret_cast<const char*>(qg + s * a.str_qk + static_cast<long long>(head) * DQ) + 16 * c;
        else if (c < 2 * per_row)
          src = reinterpret_cast<const char*>(kg + s * a.str_qk + static_cast<long long>(head) * DQ) + 16 * (c - per_row);
        else
          src = reinterpret_cast<const char*>(vg + s * a.str_v + static_cast<long long>(head) * a.DV + c0) +
                16 * (c - 2 * per_row);
        cp_async16(reinterpret_cast<char*>(dst) + 16 * c, src);
      }
    }
    cp_async_commit();
  };

  // ---- prologue --------------------------------------------------------------------------------
  float creg[Cfg::RPT];                 // compute threads: C[rows, col]
  float nreg[Cfg::RPL];                 // producer: n[prow(r)]
  float m_run = a.m_in[head];
  const int col = tid / Cfg::TPC;       // compute threads: value column in the block
  const int l = tid % Cfg::TPC;
  const float* cbase = a.c_in + static_cast<long long>(head) * DQ * a.DV + c0;

  // producer lane's n rows: pairs of adjacent rows, so q and k are read as bf16x2 / float2 words
  auto prow = [&](int r) { return 2 * lane + 64 * (r >> 1) + (r & 1); };
  if (producer) {
#pragma unroll
    for (int r = 0; r < Cfg::RPL; ++r) nreg[r] = a.n_in[head * DQ + prow(r)];
    if (blockIdx.x == 0) {
      if (a.n_save != nullptr)
#pragma unroll
        for (int r = 0; r < Cfg::RPL; ++r) a.n_save[head * DQ + prow(r)] = nreg[r];
      if (a.m_save != nullptr && lane == 0) a.m_save[head] = m_run;
    }
    for (int s = 0; s < kDepth - 1; ++s) issue(s);
    gate_chunk<T>(a, head, 0, n_steps, m_run, g_f, g_i, g_mx);
  } else if (a.stage_c) {
    // 16-byte chunk i = (row i / 4, columns 4 (i % 4) ..): a warp copies 8 whole rows per instruction. The
    // state is read and written with an L2 evict-last policy: in the decode loop it is re-read at the next
    // byte while every weight in between streams through L2 evict-first.
    const uint64_t keep = l2_evict_last_policy();
    for (int i = tid; i < DQ * 4; i += Cfg::NCOMP)
      cp_async16_hint(cst + stage_word(i >> 2, 4 * (i & 3)), cbase + static_cast<long long>(i >> 2) * a.DV + 4 * (i & 3),
                      keep);
    cp_async_commit();
    cp_async_wait<0>();
    compute_sync(Cfg::NCOMP);
#pragma unroll
    for (int ch = 0; ch < Cfg::CH; ++ch)
#pragma unroll
      for (int e = 0; e < 8; ++e) creg[ch * 8 + e] = cst[stage_word((l + Cfg::TPC * ch) * 8 + e, col)];
  } else {
#pragma unroll
    for (int ch = 0; ch < Cfg::CH; ++ch)
#pragma unroll
      for (int e = 0; e < 8; ++e) creg[ch * 8 + e] = cbase[static_cast<long long>((l + Cfg::TPC * ch) * 8 + e) * a.DV + col];
  }

  // bf16(qk_scale) in bf16 mode (Triton casts the scalar to the tensor's dtype).
  const float qsc = rnd<T>(a.qk_scale);
  float qn_prev = 0.0f;

  // ---- positions ---------------------------------------------------------------------------------
  for (int t = 0; t < n_steps; ++t) {
    if (producer) cp_async_wait<kDepth - 2>();
    __syncthreads();
    const T* st = ring[t % kDepth];
    const float fa = g_f[t & 63], ia = g_i[t & 63];
    if (producer) {
      if (want_h && t > 0 && lane < kBV) {
        const float den = __fadd_rn(fmaxf(fabsf(qn_prev), g_mx[(t - 1) & 63]), a.eps);
        static_cast<T*>(a.h)[(t - 1) * a.str_h + static_cast<long long>(head) * a.DV + c0 + lane] =
            from_f<T>(__fdiv_rn(hb[(t - 1) & 1][lane], den));
      }
      issue(t + kDepth - 1);
      float qn = 0.0f;
#pragma unroll
      for (int r = 0; r < Cfg::RPL; r += 2) {
        const int row = prow(r);
        float k0, k1, q0, q1;
        load_pair<T>(st + DQ + row, k0, k1);
        load_pair<T>(st + row, q0, q1);
        float ik0, ik1;
        mul_pair<T>(ia, k0, k1, ik0, ik1);  // i_act * k, rounded like the reference
        nreg[r] = fmaf(fa, nreg[r], ik0);
        nreg[r + 1] = fmaf(fa, nreg[r + 1], ik1);
        if (want_h) qn += dot_pair<T>(q0, q1, qsc, nreg[r], nreg[r + 1]);
      }
      if (want_h) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) qn += __shfl_xor_sync(0xffffffffu, qn, o);
        qn_prev = qn;
      }
      __syncwarp();
      if ((t & (kGC - 1)) == 0 && t + kGC < n_steps) gate_chunk<T>(a, head, t / kGC + 1, n_steps, m_run, g_f, g_i, g_mx);
    } else {
      float hs = 0.0f;
      if constexpr (sizeof(T) == 2) {
        // bf16: q, k stay packed; every product is one bf16x2 multiply rounded to nearest (the
        // reference's bf16 x bf16 products), the state update and the sum are fp32.
        const __nv_bfloat162 v2 = __bfloat162bfloat162(st[2 * DQ + col]);
        const __nv_bfloat162 ia2 = pack2(ia, ia), qsc2 = pack2(qsc, qsc);
#pragma unroll
        for (int ch = 0; ch < Cfg::CH; ++ch) {
          const int rb = (l + Cfg::TPC * ch) * 8;
          const uint4 kw = *reinterpret_cast<const uint4*>(st + DQ + rb);
          const uint4 qw = *reinterpret_cast<const uint4*>(st + rb);
          const __nv_bfloat162* k2 = reinterpret_cast<const __nv_bfloat162*>(&kw);
          const __nv_bfloat162* q2 = reinterpret_cast<const __nv_bfloat162*>(&qw);
#pragma unroll
          for (int p = 0; p < 4; ++p) {
            float& c0 = creg[ch * 8 + 2 * p];
            float& c1 = creg[ch * 8 + 2 * p + 1];
            float u0, u1;
            unpack2(__hmul2(ia2, __hmul2(k2[p], v2)), u0, u1);
            c0 = fmaf(fa, c0, u0);
            c1 = fmaf(fa, c1, u1);
            if (want_h) {
              float p0, p1;
              unpack2(__hmul2(__hmul2(q2[p], qsc2), __floats2bfloat162_rn(c0, c1)), p0, p1);
              hs += p0 + p1;
            }
          }
        }
      } else {
        const float vf = to_f<T>(st[2 * DQ + col]);
#pragma unroll
        for (int ch = 0; ch < Cfg::CH; ++ch) {
          const int rb = (l + Cfg::TPC * ch) * 8;
          const float4* kp = reinterpret_cast<const float4*>(st + DQ + rb);
          const float4* qp = reinterpret_cast<const float4*>(st + rb);
          const float4 ka = kp[0], kb = kp[1], qa = qp[0], qb = qp[1];
          const float kf[8] = {ka.x, ka.y, ka.z, ka.w, kb.x, kb.y, kb.z, kb.w};
          const float qf[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            float& c = creg[ch * 8 + e];
            c = fmaf(fa, c, ia * (kf[e] * vf));
            if (want_h) hs += (qf[e] * qsc) * c;
          }
        }
      }
      if (want_h) {
#pragma unroll
        for (int o = Cfg::TPC / 2; o > 0; o >>= 1) hs += __shfl_xor_sync(0xffffffffu, hs, o);
        if (l == 0) hb[t & 1][col] = hs;
      }
    }
  }
  // ---- epilogue -----------------------------------------------------------------------------------
  // The compute threads write C first (it needs nothing from the producer), so that the stores are
  // under way while the barrier below hands the producer the last position's h sums.
  if (!producer && a.c_out != nullptr) {
    float* obase = a.c_out + static_cast<long long>(head) * DQ * a.DV + c0;
    if (a.stage_c) {
#pragma unroll
      for (int ch = 0; ch < Cfg::CH; ++ch)
#pragma unroll
        for (int e = 0; e < 8; ++e) cst[stage_word((l + Cfg::TPC * ch) * 8 + e, col)] = creg[ch * 8 + e];
      compute_sync(Cfg::NCOMP);
      const uint64_t keep = l2_evict_last_policy();
      for (int i = tid; i < DQ * 4; i += Cfg::NCOMP)
        st_global16_hint(obase + static_cast<long long>(i >> 2) * a.DV + 4 * (i & 3),
                         *reinterpret_cast<const float4*>(cst + stage_word(i >> 2, 4 * (i & 3))), keep);
    } else {
#pragma unroll
      for (int ch = 0; ch < Cfg::CH; ++ch)
#pragma unroll
        for (int e = 0; e < 8; ++e) obase[static_cast<long long>((l + Cfg::TPC * ch) * 8 + e) * a.DV + col] = creg[ch * 8 + e];
    }
  }
  cp_async_wait<0>();
  __syncthreads();
  if (producer) {
    if (want_h && n_steps > 0 && lane < kBV) {
      const int t = n_steps - 1;
      const float den = __fadd_rn(fmaxf(fabsf(qn_prev), g_mx[t & 63]), a.eps);
      static_cast<T*>(a.h)[t * a.str_h + static_cast<long long>(head) * a.DV + c0 + lane] =
          from_f<T>(__fdiv_rn(hb[t & 1][lane], den));
    }
    if (blockIdx.x == 0) {
      if (a.n_out != nullptr)
#pragma unroll
        for (int r = 0; r < Cfg::RPL; ++r) a.n_out[head * DQ + prow(r)] = nreg[r];
      if (a.m_out != nullptr && lane == 0) a.m_out[head] = m_run;
    }
  }
}

__global__ void accept_kernel(const int64_t* ids, const int64_t* tok, int64_t* out, int S, int smax) {
  pdl_launch_dependents();
  pdl_wait_prior_grids();
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  int64_t alive = 1, n = 0;
  for (int j = 0; j < S - 1; ++j) {
    alive = alive && (ids[1 + j] == tok[j]);
    n += alive;
  }
  for (int j = 0; j < S; ++j) out[j] = tok[j];
  out[smax] = n;
}

// State commit of the drafting loop: cur <- hist[slot] for the three tensors of one layer's state, the slot
// (the accepted length) read on the device so that a CUDA graph replays the commit for whatever length the
// round accepted. Segment j copies cnt[j] floats from src[j] + slot * cnt[j] to dst[j]; 16-byte copies when
// every address and count allows, single floats otherwise. A slot outside [0, slots) fills cur with NaN and
// reads nothing.
struct CommitArgs {
  const float* src[3];
  float* dst[3];
  long long cnt[3];
  const void* slot;
  int slot_bytes;  // 4 (int32) or 8 (int64)
  int slots;
  int vec;  // 1: 16-byte copies
};

__global__ void __launch_bounds__(256) commit_state_kernel(const CommitArgs a) {
  pdl_launch_dependents();
  pdl_wait_prior_grids();
  const long long slot = a.slot_bytes == 8 ? *static_cast<const long long*>(a.slot)
                                           : static_cast<long long>(*static_cast<const int*>(a.slot));
  const bool ok = slot >= 0 && slot < a.slots;
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
  const long long t0 = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
#pragma unroll
  for (int j = 0; j < 3; ++j) {
    const long long n = a.cnt[j];
    if (n == 0) continue;
    float* d = a.dst[j];
    if (!ok) {
      for (long long e = t0; e < n; e += stride) d[e] = __int_as_float(0x7fc00000);
      continue;
    }
    const float* sp = a.src[j] + slot * n;
    if (a.vec) {
      const float4* s4 = reinterpret_cast<const float4*>(sp);
      float4* d4 = reinterpret_cast<float4*>(d);
      for (long long e = t0; e < n / 4; e += stride) d4[e] = __ldcs(s4 + e);
    } else {
      for (long long e = t0; e < n; e += stride) d[e] = sp[e];
    }
  }
}

// Opts the kernel into `bytes` of dynamic shared memory, once per device.
template <typename K>
int allow_dynamic_smem(K kernel, size_t bytes, bool* done) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return fail(BP_ERR_CUDA, "cudaGetDevice failed");
  if (done[dev]) return BP_OK;
  const cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(bytes));
  if (e != cudaSuccess) return fail(BP_ERR_CUDA, "cudaFuncSetAttribute(smem %zu): %s", bytes, cudaGetErrorString(e));
  done[dev] = true;
  return BP_OK;
}

template <int DQ, typename T>
int launch_scan(const ScanArgs& a, cudaStream_t s) {
  using Cfg = ScanCfg<DQ, T>;
  dim3 grid(a.DV / kBV, a.NH, 1);
  const size_t smem = a.stage_c ? static_cast<size_t>(DQ) * kBV * sizeof(float) : 0;
  static bool attr_done[64] = {};
  if (smem > 0) {
    const int st = allow_dynamic_smem(mlstm_scan_kernel<DQ, T>, smem, attr_done);
    if (st != BP_OK) return st;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(Cfg::NTHREADS, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  set_launch_attrs(cfg, attr);
  const cudaError_t e = cudaLaunchKernelEx(&cfg, mlstm_scan_kernel<DQ, T>, a);
  if (e != cudaSuccess) return fail(BP_ERR_CUDA, "mlstm scan launch: %s", cudaGetErrorString(e));
  return BP_OK;
}

template <typename T>
int dispatch_dq(const ScanArgs& a, int DQ, cudaStream_t s) {
  switch (DQ) {
    case 64: return launch_scan<64, T>(a, s);
    case 128: return launch_scan<128, T>(a, s);
    case 256: return launch_scan<256, T>(a, s);
    case 512: return launch_scan<512, T>(a, s);
    default: return fail(BP_ERR_UNSUPPORTED, "head dim DQ = %d is not one of 64, 128, 256, 512", DQ);
  }
}

bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace
}  // namespace bp

extern "C" int bp_mlstm_scan(const float* c_in, const float* n_in, const float* m_in, const void* q, const void* k,
                             const void* v, const void* i_gate, const void* f_gate, void* h, float* c_out, float* n_out,
                             float* m_out, float* n_save, float* m_save, const int64_t* steps_dev, int T, int NH, int DQ,
                             int DV, long long str_t_qk, long long str_t_v, long long str_t_if, long long str_t_h,
                             int dtype, int gate_dtype, float qk_scale, float eps, void* stream) {
  using namespace bp;
  clear_error();
  if (T < 0 || NH <= 0 || DQ <= 0 || DV <= 0) return fail(BP_ERR_INVALID_ARGUMENT, "bad sizes T=%d NH=%d DQ=%d DV=%d", T, NH, DQ, DV);
  if (dtype != BP_DTYPE_BF16 && dtype != BP_DTYPE_F32) return fail(BP_ERR_INVALID_ARGUMENT, "dtype %d is not bf16 or fp32", dtype);
  if (gate_dtype != BP_DTYPE_BF16 && gate_dtype != BP_DTYPE_F32)
    return fail(BP_ERR_INVALID_ARGUMENT, "gate dtype %d is not bf16 or fp32", gate_dtype);
  if (DV % kBV != 0) return fail(BP_ERR_UNSUPPORTED, "DV = %d is not a multiple of %d", DV, kBV);
  if (c_in == nullptr || n_in == nullptr || m_in == nullptr) return fail(BP_ERR_INVALID_ARGUMENT, "start state is NULL");
  if (T > 0 && (q == nullptr || k == nullptr || v == nullptr || i_gate == nullptr || f_gate == nullptr))
    return fail(BP_ERR_INVALID_ARGUMENT, "q, k, v, i or f is NULL");
  if ((n_out != nullptr && n_out == n_in) || (m_out != nullptr && m_out == m_in))
    return fail(BP_ERR_INVALID_ARGUMENT, "n_out / m_out must not alias n_in / m_in (other CTAs still read them)");
  const int vec_elems = dtype == BP_DTYPE_BF16 ? 8 : 4;
  if (!al16(q) || !al16(k) || !al16(v) || str_t_qk % vec_elems || str_t_v % vec_elems)
    return fail(BP_ERR_MISALIGNED, "q/k/v need 16-byte aligned bases and position strides that are multiples of %d elements",
                vec_elems);
  if (T > 0 && (str_t_qk < static_cast<long long>(NH) * DQ || str_t_v < static_cast<long long>(NH) * DV || str_t_if < NH ||
                (h != nullptr && str_t_h < static_cast<long long>(NH) * DV)))
    return fail(BP_ERR_INVALID_ARGUMENT, "a position stride is smaller than one position");
  int st = require_sm100();
  if (st != BP_OK) return st;
  ScanArgs a;
  a.c_in = c_in; a.n_in = n_in; a.m_in = m_in;
  a.q = q; a.k = k; a.v = v; a.ig = i_gate; a.fg = f_gate; a.h = h;
  a.c_out = c_out; a.n_out = n_out; a.m_out = m_out; a.n_save = n_save; a.m_save = m_save;
  a.steps_dev = steps_dev;
  a.T = T; a.NH = NH; a.DV = DV;
  a.str_qk = str_t_qk; a.str_v = str_t_v; a.str_if = str_t_if; a.str_h = str_t_h;
  a.gate_f32 = gate_dtype == BP_DTYPE_F32;
  a.stage_c = al16(c_in) && (c_out == nullptr || al16(c_out));
  a.qk_scale = qk_scale; a.eps = eps;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return dtype == BP_DTYPE_BF16 ? dispatch_dq<__nv_bfloat16>(a, DQ, s) : dispatch_dq<float>(a, DQ, s);
}

extern "C" int bp_mlstm_accept(const int64_t* ids, const int64_t* tok, int64_t* out, int S, int smax, void* stream) {
  using namespace bp;
  clear_error();
  if (S < 0 || smax < S) return fail(BP_ERR_INVALID_ARGUMENT, "need 0 <= S <= smax (S=%d smax=%d)", S, smax);
  if (ids == nullptr || tok == nullptr || out == nullptr) return fail(BP_ERR_INVALID_ARGUMENT, "NULL pointer");
  int st = require_sm100();
  if (st != BP_OK) return st;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(1, 1, 1);
  cfg.blockDim = dim3(32, 1, 1);
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[2];
  set_launch_attrs(cfg, attr);
  const cudaError_t e = cudaLaunchKernelEx(&cfg, accept_kernel, ids, tok, out, S, smax);
  if (e != cudaSuccess) return fail(BP_ERR_CUDA, "accept launch: %s", cudaGetErrorString(e));
  return BP_OK;
}

// Counterpart of byteprof/optim/draft_core.py:92-111 (commit_state and its Triton commit_kernel,
// byteprof/optim/draft_kernels.py:7-18).
extern "C" int bp_mlstm_commit_state(const float* c_hist, const float* n_hist, const float* m_hist, float* c_cur,
                                     float* n_cur, float* m_cur, long long c_count, long long n_count, long long m_count,
                                     const void* slot, int slot_bytes, int slots, void* stream) {
  using namespace bp;
  clear_error();
  if (c_count < 0 || n_count < 0 || m_count < 0 || slots <= 0)
    return fail(BP_ERR_INVALID_ARGUMENT, "negative count or no history slots");
  if (slot_bytes != 4 && slot_bytes != 8) return fail(BP_ERR_INVALID_ARGUMENT, "slot must be int32 or int64");
  if (slot == nullptr) return fail(BP_ERR_INVALID_ARGUMENT, "slot is NULL");
  if ((c_count > 0 && (c_hist == nullptr || c_cur == nullptr)) || (n_count > 0 && (n_hist == nullptr || n_cur == nullptr)) ||
      (m_count > 0 && (m_hist == nullptr || m_cur == nullptr)))
    return fail(BP_ERR_INVALID_ARGUMENT, "NULL state pointer");
  int st = require_sm100();
  if (st != BP_OK) return st;
  CommitArgs a;
  a.src[0] = c_hist; a.src[1] = n_hist; a.src[2] = m_hist;
  a.dst[0] = c_cur; a.dst[1] = n_cur; a.dst[2] = m_cur;
  a.cnt[0] = c_count; a.cnt[1] = n_count; a.cnt[2] = m_count;
  a.slot = slot;
  a.slot_bytes = slot_bytes;
  a.slots = slots;
  a.vec = 1;
  for (int j = 0; j < 3; ++j)
    if (a.cnt[j] % 4 != 0 || !al16(a.src[j]) || !al16(a.dst[j])) a.vec = 0;
  long long most = c_count > n_count ? c_count : n_count;
  most = most > m_count ? most : m_count;
  long long blocks = (most / (a.vec ? 4 : 1) + 255) / 256;
  blocks = blocks < 1 ? 1 : (blocks > 4 * 148 ? 4 * 148 : blocks);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(blocks), 1, 1);
  cfg.blockDim = dim3(256, 1, 1);
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[2];
  set_launch_attrs(cfg, attr);
  const cudaError_t e = cudaLaunchKernelEx(&cfg, commit_state_kernel, a);
  if (e != cudaSuccess) return fail(BP_ERR_CUDA, "commit state launch: %s", cudaGetErrorString(e));
  return BP_OK;
}
