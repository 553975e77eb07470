/*
 * bp_kernels.h -- C ABI of the B200 (sm_100a) kernels behind byteprof's decode hot path.
 *
 * Every entry point takes caller-owned device pointers, plain integer sizes and strides, and a
 * cudaStream_t passed as `void*` (NULL = the legacy default stream). Nothing here allocates device
 * memory, synchronises the host or aborts: each call returns a status (BP_OK = 0), and
 * bp_last_error() returns a message for the last failing call on the calling thread. All launches
 * go to the given stream, so the calls can be captured in a CUDA graph.
 *
 * Reference interfaces replaced (paths inside the byteprof project):
 *   bp_skinny_mm        byteprof/optim/skinny.py:136-166   skinny_mm (bf16 and int8 weight kinds)
 *                       byteprof/optim/skinny.py:111-129   _launch (+ _split_reduce, skinny.py:83-90)
 *   bp_gemv_int8        byteprof/quant/triton_int8.py:40-47 gemv_int8
 *   bp_skinny_mm_int4   byteprof/optim/skinny.py:46-63, 136-166 skinny_mm (int4 g128 weight kind)
 *   bp_rmsnorm          byteprof/optim/bolmo_draft.py:74-100 the local layers' norms (K + 1 rows)
 *   bp_mlstm_scan       byteprof/optim/mlstm_multistep.py:33-85  multistep_fw_kernel
 *                       byteprof/optim/mlstm_multistep.py:89-133 lazy_commit_kernel
 *                       byteprof/optim/draft_core.py:114-141     mlstm_step_into (library step)
 *   bp_mlstm_accept     byteprof/optim/mlstm_multistep.py:136-146 accept_kernel
 *   bp_mlstm_commit_state byteprof/optim/draft_core.py:92-111  commit_state (+ draft_kernels.py commit_kernel)
 *   bp_rmsnorm_ex, bp_embed_rmsnorm, bp_swiglu, bp_gate_softcap, bp_decode_attention, bp_decode_finish, bp_glob_step,
 *   bp_loc_enc_step, bp_loc_dec_step, bp_loc_encdec_step
 *                       the per-byte pieces of the minimal Bolmo loop: byteprof/optim/bolmo.py:32-136
 *                       (_layer_step, LocalLoop.enc_step / dec_step, GlobalStep.step) and
 *                       byteprof/optim/bolmo_loop.py:36-64 (MinimalPieces: norm, lm_head, argmax)
 */
#ifndef BP_KERNELS_H
#define BP_KERNELS_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ------------------------------------------------------------------------- */
enum {
  BP_OK = 0,
  BP_ERR_INVALID_ARGUMENT = 1, /* a size, stride, pointer or dtype is not accepted */
  BP_ERR_UNSUPPORTED = 2,      /* a valid request this build has no kernel for (e.g. head dim) */
  BP_ERR_MISALIGNED = 3,       /* a pointer or stride breaks the alignment the kernel needs */
  BP_ERR_CUDA = 4,             /* the CUDA runtime reported an error (launch or device) */
  BP_ERR_NO_DEVICE = 5         /* no sm_100 device is current */
};

/* ---- element types ------------------------------------------------------------------------ */
enum {
  BP_DTYPE_BF16 = 0,
  BP_DTYPE_F32 = 1,
  BP_DTYPE_INT8 = 2,
  BP_DTYPE_INT4 = 3 /* byteprof's tile-major int4 group-128 format (bp_skinny_mm_int4) */
};

/* Version of this ABI (major * 100 + minor). */
int bp_abi_version(void);

/* Human-readable name of a status code (static storage). */
const char* bp_status_string(int status);

/* Message describing the last failing call on this thread ("" when none). */
const char* bp_last_error(void);

/*
 * Skinny linear  y[M, N] = x[M, K] . W[N, K]^T  (fp32 accumulation).
 *   x      bf16, row stride ldx elements (ldx >= K); rows beyond M are never read
 *   w      w_dtype = BP_DTYPE_BF16: bf16 [N, K] contiguous
 *          w_dtype = BP_DTYPE_INT8: int8 [N, K] contiguous, w_scale = bf16 [N]; y = scale[n] * sum_k x*q.
 *          Aligned int8 problems (x and w 16-byte aligned, ldx a multiple of 8, K a multiple of 16) sum
 *          exactly over x written in fixed point (29 bits below each row's largest exponent: every x within
 *          2^-22 of the row maximum is exact) and round scale * sum once, on the tensor cores or, for one
 *          row and at most 4096 output rows, on the CUDA cores in one launch: the two give the same
 *          bits, so a row's result never depends on M. A row of x holding Inf or NaN gives a NaN row of y
 *   y      y_dtype BP_DTYPE_BF16 or BP_DTYPE_F32 (the fp32 store is the un-rounded accumulator), row
 *          stride ldy elements; exactly the M x N block is written
 *   workspace, workspace_bytes  caller-owned device scratch of at least
 *          bp_skinny_workspace_bytes(M, N, K, w_dtype) bytes, 256-byte aligned, zero-filled once before
 *          its first use; every call leaves it zero-filled again. Calls that overlap in time (other
 *          streams) must use different workspaces. May be NULL when the query returns 0.
 * M = 0 or N = 0 writes nothing; K = 0 writes zeros. Any M is accepted; rows are processed in
 * chunks of 16 per launch (the weights are re-read per chunk, as the reference re-reads per 64 rows).
 * Replaces skinny_mm / _launch / _skinny_kernel MODE 0 and 1 (byteprof/optim/skinny.py:35-166).
 */
int bp_skinny_mm(const void* x, long long ldx, const void* w, int w_dtype, const void* w_scale,
                 void* y, long long ldy, int y_dtype, int M, int N, int K, void* workspace,
                 size_t workspace_bytes, void* stream);

/*
 * Workspace bytes bp_skinny_mm (w_dtype BP_DTYPE_BF16 or BP_DTYPE_INT8) or bp_skinny_mm_int4
 * (w_dtype BP_DTYPE_INT4) needs for this problem on the current device (0: none needed). The
 * stream-K partial sums of the tensor-core paths live there (int8 and int4: also the activations'
 * digit planes, 64 K bytes; int8: exact int64 partials, about 9.5 MB on 148 SMs;
 * byteprof/optim/skinny.py:125 allocates its split-K workspace per call instead).
 */
size_t bp_skinny_workspace_bytes(int M, int N, int K, int w_dtype);

/*
 * bp_skinny_mm for callers that cannot allocate device memory (no counterpart in the reference).
 * Same arguments and results as bp_skinny_mm without the workspace: the scratch of the
 * tensor-core path (bf16 and int8 weights) is a fixed 11.6 MB array inside the library (held by every GPU that loads it, until
 * the process exits). Meant for code that runs during CUDA-graph capture in global mode, where
 * cudaMalloc is refused, and for hosts that give their plugins no allocator.
 * Limits: N <= 1,048,576 rows, K <= 16384 for int8 weights and a device with at most 160 SMs; larger problems return
 * BP_ERR_UNSUPPORTED. Allocates nothing. The first call on a device looks up the array's device
 * address (cudaGetSymbolAddress): make that first call before any stream capture. Each call clears the
 * array's tile counters on the stream, then launches; every call shares the one array, so calls that
 * overlap on the GPU (other streams) race with each other.
 */
int bp_skinny_mm_static_scratch(const void* x, long long ldx, const void* w, int w_dtype, const void* w_scale,
                                void* y, long long ldy, int y_dtype, int M, int N, int K, void* stream);

/*
 * Skinny linear with fp32 activations: bp_skinny_mm's arithmetic (the CUDA-core kernel: the K partition
 * depends on N and K only, fp32 accumulation) with x read as fp32 [M, K] (16-byte aligned and ldx a
 * multiple of 4 for the vector path). Weights bf16 or int8 + bf16 scale, y bf16 or fp32, no workspace.
 * No counterpart in the reference, whose fp32 activations go to F.linear on dequantized fp32 weights
 * (byteprof/optim/skinny_linear.py:67-68): it serves the byte decoder's fp32-activation exactness mode.
 */
int bp_skinny_mm_xf32(const float* x, long long ldx, const void* w, int w_dtype, const void* w_scale, void* y,
                      long long ldy, int y_dtype, int M, int N, int K, void* stream);

/*
 * int8 weight-only GEMV for one activation row: y[1, N] = scale[n] * sum_k x[k] * q[n, k].
 * bp_skinny_mm with M = 1 and int8 weights, including its workspace rule and its results, bit for bit
 * (byteprof/quant/triton_int8.py:15-47).
 */
int bp_gemv_int8(const void* x, const int8_t* w, const void* w_scale, void* y, int y_dtype, int N, int K,
                 void* workspace, size_t workspace_bytes, void* stream);

/*
 * Skinny linear with int4 weights in groups of 128 along K, in byteprof's tile-major format:
 *   y[m, n] = sum_g scale[g, n] * sum_{k in group g} (q[n, k] - zero[g, n]) * x[m, k].
 *   w_packed  uint8 [ceil(N / tile_rows), K / 128, tile_rows, 64]: inside a group, byte j of a row holds
 *             code j (low nibble) and code j + 64 (high nibble); padding rows are zero
 *   scale     bf16 [K / 128, N];  zero  fp16 [K / 128, N]
 *   x         bf16, 16-byte aligned, ldx a multiple of 8; y as in bp_skinny_mm (bf16 or fp32)
 *   workspace, workspace_bytes  as in bp_skinny_mm, sized by bp_skinny_workspace_bytes(M, N, K,
 *             BP_DTYPE_INT4); NULL with 0 bytes selects the CUDA-core kernel, which needs none
 * K must be a multiple of 128 and tile_rows 32 (the format's default; other values return
 * BP_ERR_UNSUPPORTED). Any M (16 rows per launch). With a workspace, N a multiple of 8 and scale and
 * zero 16-byte aligned, the tensor-core kernel runs: x written exactly as fixed point (as for int8
 * weights), exact integer group sums, a row of x holding Inf or NaN gives a NaN row of y. Otherwise
 * the CUDA-core kernel runs (split-K partials meet in distributed shared memory). Either way a row's
 * result does not depend on M or on the other rows. Replaces skinny_mm with uint8 weights /
 * _skinny_kernel MODE 3 (byteprof/optim/skinny.py:1-19, 46-63, 136-166).
 */
int bp_skinny_mm_int4(const void* x, long long ldx, const uint8_t* w_packed, const void* scale, const void* zero,
                      void* y, long long ldy, int y_dtype, int M, int N, int K, int tile_rows, void* workspace,
                      size_t workspace_bytes, void* stream);

/*
 * Row-wise RMSNorm, bf16 in and out, fp32 arithmetic: y[r, :] = x[r, :] * rsqrt(mean(x[r, :]^2) + eps) * w.
 * One warp per row with a fixed summation order, so a row's result does not depend on how many rows
 * the call holds (verifying K drafts at once gives the bits of K single steps). cols a multiple of 8,
 * rows 16-byte aligned, strides multiples of 8 elements. Replaces the pre-norms, the per-head output
 * norm and the final norm of the local layers run by byteprof's drafting engine
 * (byteprof/optim/bolmo_draft.py:74-100).
 */
int bp_rmsnorm(const void* x, long long ldx, const void* w, void* y, long long ldy, int rows, int cols, float eps,
               void* stream);

/*
 * RMSNorm fused with the step around it, one warp per row with bp_rmsnorm's summation order. x, res,
 * s_out and y hold `dtype` values (BP_DTYPE_BF16 or BP_DTYPE_F32), w is bf16, arithmetic fp32. With bf16
 * every step rounds where a bf16 tensor would hold the value (as written below); with fp32 nothing is
 * rounded to bf16. n(v) = bf16(v * rsqrt(mean(v^2) + eps) * w):
 *   BP_NORM_PLAIN      y = n(x)
 *   BP_NORM_ADD_FIRST  s = bf16(x + res); y = n(s)     (s_out receives s when not NULL)
 *   BP_NORM_ADD_AFTER  y = bf16(res + n(x))
 *   BP_NORM_GATE       y = bf16(bf16(sigmoid(res)) * n(x))
 * Rows come in groups of w_rows, the rows of w ([w_rows, cols]): row r = g * w_rows + j uses weight
 * row j and lives at element g * ld + j * cols of x, res, s_out and y (w_rows = 1: row r at r * ld).
 * ldres = 0 broadcasts one res row. cols and strides multiples of 8, 16-byte aligned bases.
 * Replaces the RMSNorm + residual add, RMSNorm + add (OLMo-2) and output-gate steps of the layers the
 * minimal Bolmo loop runs (byteprof/optim/bolmo.py:32-44, 100-136).
 */
enum { BP_NORM_PLAIN = 0, BP_NORM_ADD_FIRST = 1, BP_NORM_ADD_AFTER = 2, BP_NORM_GATE = 3 };
int bp_rmsnorm_ex(const void* x, long long ldx, const void* w, int w_rows, const void* res, long long ldres,
                  void* s_out, long long lds, void* y, long long ldy, int rows, int cols, float eps, int mode,
                  int dtype, void* stream);

/*
 * Embedding lookup + RMSNorm, bf16: h_out[r] = table[index[r]] (h_out may be NULL) and
 * y[r] = bf16(h_out[r] * rsqrt(mean(h_out[r]^2) + eps) * w) for r < rows; index int64 on the device, an
 * index outside [0, table_rows) gives NaN rows. cols and strides multiples of 8, 16-byte aligned bases.
 * Replaces the byte embedding of the local encoder and its layer's first norm (byteprof/optim/bolmo.py:
 * 82-90, LocalLoop.enc_step: enc._embed, then the layer's pre-norm) in one launch. Added with ABI
 * version 201.
 */
int bp_embed_rmsnorm(const void* table, long long ld_table, long long table_rows, const int64_t* index, const void* w,
                     void* h_out, long long ldh, void* y, long long ldy, int rows, int cols, float eps, void* stream);

/*
 * SwiGLU: out[r, j] = bf16(bf16(silu(gu[r, j])) * gu[r, ffn + j]) for j < ffn (gate | up halves of one
 * GEMM output) with dtype BP_DTYPE_BF16; with BP_DTYPE_F32 gu and out are fp32 and nothing is rounded to
 * bf16. ffn and strides multiples of 8, 16-byte aligned. Replaces act_fn(gate) * up of the MLPs in the
 * Bolmo layers (byteprof/optim/bolmo.py:32-44).
 */
int bp_swiglu(const void* gu, long long ldgu, void* out, long long ldo, int rows, int ffn, int dtype, void* stream);

/*
 * mLSTM gate pre-activations: out[r, c] = cap * tanh((g[r, c] + bias[c]) / cap), fp32 (bias may be
 * NULL; out may equal g). Replaces the soft cap of the xLSTM layer's input / forget gates.
 */
int bp_gate_softcap(const float* g, long long ldg, const float* bias, float* out, long long ldo, int rows, int n,
                    float cap, void* stream);

/*
 * One query position of an OLMo-2 attention layer against a static KV cache, position p = *pos read on
 * the device (so a CUDA graph replays it at every position):
 *   qkv [3 * nh * head_dim] bf16 = q | k | v of the position; q and k are RMS-normalised over the
 *   whole width (weights q_norm_w, k_norm_w, eps), rotated (rotary halves; cos_t / sin_t fp32
 *   [max_pos, head_dim / 2]), k and v written to k_cache / v_cache [max_pos, nh, head_dim] bf16 at p;
 *   out [nh * head_dim] bf16 = softmax(q . k_j * scale) over j <= p, times v_j.
 * Work per head is one thread-block cluster of 8 CTAs (128 positions each per 1024-position round),
 * merged in the leader CTA in a fixed order (deterministic). head_dim 128. A position outside
 * [0, max_pos) writes NaN and touches no cache row. dtype BP_DTYPE_BF16 as above; BP_DTYPE_F32: qkv,
 * the caches and out hold fp32 values and nothing is rounded to bf16.
 * Replaces GlobalStep.step's attention over the StaticCache (byteprof/optim/bolmo.py:100-136).
 */
int bp_decode_attention(const void* qkv, const void* q_norm_w, const void* k_norm_w, const float* cos_t,
                        const float* sin_t, const int64_t* pos, void* k_cache, void* v_cache, void* out, int nh,
                        int head_dim, int max_pos, float eps, float scale, int dtype, void* stream);

/*
 * One global-model step of a Bolmo-1B-shaped byte decoder in a single persistent (cooperative) kernel:
 * n_layers OLMo-2 blocks (d 2048, 16 heads x 128, SwiGLU 8192; RMSNorm of q and k over d, rotary
 * embedding, attention over the static KV caches, RMSNorm of the attention and MLP outputs before each
 * residual add) at patch position p = *pos, then value_out = rmsnorm(x_L) * out_norm and *pos = p + 1.
 * Per layer: w_qkv [3d, d], q_norm [d], k_norm [d], w_o [d, d], attn_norm [d], w_gu [2 ffn, d] (gate rows,
 * then up rows), w_down [d, ffn], mlp_norm [d], k_cache / v_cache [max_pos, 16, 128]; all bf16, 16-byte
 * aligned. cos_t / sin_t fp32 [max_pos, 64]. workspace: the size bp_glob_step_workspace_bytes returns,
 * 16-byte aligned, zero-filled before its first launch and not written by anything else afterwards (it
 * carries a launch number from one launch to the next; ABI version 202 added this requirement). Calls
 * sharing a workspace must not overlap. Results equal the kernel-by-kernel path (bp_skinny_mm, bp_decode_attention,
 * bp_rmsnorm_ex, bp_swiglu) up to the summation order of the matrix-vector products. Not capturable
 * together with other work that needs the SMs meanwhile (one CTA per SM, all resident). Replaces
 * GlobalStep.step (byteprof/optim/bolmo.py:100-136).
 */
typedef struct bp_glob_layer {
  const void* w_qkv;
  const void* q_norm;
  const void* k_norm;
  const void* w_o;
  const void* attn_norm;
  const void* w_gu;
  const void* w_down;
  const void* mlp_norm;
  void* k_cache;
  void* v_cache;
} bp_glob_layer;
/*
 * The per-byte host loop of the byte decoder (no reference counterpart in C: byteprof/optim/bolmo_loop.py:
 * 182-207 runs it in Python). graph_execs: four cudaGraphExec_t, index 2 * parity + patch, each running one
 * whole byte: copy *byte_host in, the steps, copy (token, boundary flag) to out_host[0..1]. Step i feeds
 * bytes[i] (or, when bytes is NULL, first_byte at step 0 and then the previous step's token) with patch
 * start patches[i] (or first_patch, then the previous step's flag), launches the graph on `stream`, waits
 * for it and stores the token and flag in tokens_out[i], flags_out[i]; parity alternates from `parity`.
 * byte_host and out_host are pinned host memory; wall_seconds (may be NULL) gets the loop's wall time.
 * Added with ABI version 203.
 */
int bp_decode_loop(void* const* graph_execs, int64_t* byte_host, const int64_t* out_host, const int64_t* bytes,
                   const int32_t* patches, int n, int64_t first_byte, int32_t first_patch, int parity,
                   int64_t* tokens_out, int32_t* flags_out, void* stream, double* wall_seconds);

size_t bp_glob_step_workspace_bytes(void);
int bp_glob_step(const bp_glob_layer* layers, int n_layers, const void* x_in, const void* out_norm, void* value_out,
                 int64_t* pos, const float* cos_t, const float* sin_t, int max_pos, float eps, void* workspace,
                 size_t workspace_bytes, void* stream);

/*
 * One local step of a Bolmo-shaped byte decoder (d 2048; mLSTM 4 heads x 512; SwiGLU 2816; vocabulary 512)
 * in a single persistent (cooperative) kernel. The layer: x = rmsnorm(h) * norm1; y = w_qkvo x (q | k | v |
 * o, [4d, d]); g = cap * tanh((w_if x + b_if) / cap) ([2 NH, d], b_if fp32; input gates then forget gates);
 * the mLSTM step on the state c [NH, 512, 512] (in place) and n [NH, 512], m [NH] (fp32, read from
 * n_cur / m_cur, written to n_next / m_next); z = sigmoid(o) * rmsnorm_head(h_mlstm) * mh_norm [NH, 512];
 * h2 = h + w_out z; output = h2 + w_down (silu(W_gate x2) * W_up x2), x2 = rmsnorm(h2) * norm2, w_gu
 * [2 * 2816, d] (gate rows, then up rows), w_down [d, 2816]. All weights bf16, 16-byte aligned. Each
 * call needs the workspace size bp_loc_step_workspace_bytes returns (16-byte aligned, zero-filled before
 * its first launch and then left to the kernel: it carries the launch number from one call to the next)
 * and the whole GPU while it runs. Changed with ABI version 204 (the workspace was scratch before).
 *   bp_loc_enc_step: h = embed[*byte] (embed [512, d]); e_out = rmsnorm(output) * enc_norm; patch_out =
 *     w_patch e (bf16 [d]); *boundary_logit = w_boundary . e (fp32; w_boundary [1, d]). A byte outside
 *     [0, 512) writes NaN and leaves the state alone.
 *   bp_loc_dec_step: h = bf16(w_in e_in + value); logits = lm_head (rmsnorm(output) * final_norm) (fp32
 *     [512]); out[0] = argmax(logits) (torch order), out[1] = sigmoid(*boundary_logit) >= 0.5.
 * Results equal the kernel-by-kernel step (bp_skinny_mm, bp_rmsnorm_ex, bp_gate_softcap, bp_mlstm_scan,
 * bp_swiglu) except for summation orders. Replaces LocalLoop.enc_step / dec_step with the norm, out
 * projection, LM head and argmax of MinimalPieces (byteprof/optim/bolmo.py:32-97, bolmo_loop.py:36-64).
 */
typedef struct bp_loc_layer {
  const void* norm1;
  const void* w_qkvo;
  const void* w_if;
  const float* b_if;
  const void* mh_norm;
  const void* w_out;
  const void* norm2;
  const void* w_gu;
  const void* w_down;
  float* c;
  const float* n_cur;
  const float* m_cur;
  float* n_next;
  float* m_next;
} bp_loc_layer;
size_t bp_loc_step_workspace_bytes(void);
int bp_loc_enc_step(const bp_loc_layer* layer, const void* embed, const int64_t* byte, const void* enc_norm,
                    const void* w_patch, const void* w_boundary, void* e_out, void* patch_out, float* boundary_logit,
                    float eps, float gate_cap, float mlstm_eps, void* workspace, size_t workspace_bytes, void* stream);
int bp_loc_dec_step(const bp_loc_layer* layer, const void* e_in, const void* value, const void* w_in,
                    const void* final_norm, const void* lm_head, const float* boundary_logit, float* logits,
                    int64_t* out, float eps, float gate_cap, float mlstm_eps, void* workspace, size_t workspace_bytes,
                    void* stream);
/*
 * bp_loc_encdec_step: bp_loc_enc_step and then bp_loc_dec_step of the same byte (e_in = e_out, the encoder's
 * boundary logit for the decision) in one persistent launch, for a byte that opens no patch (the global
 * step does not run between them): the decoder's weights stream into the ring while the encoder finishes,
 * and one launch boundary goes. Results equal the two launches bit for bit. The workspace is the encoder's
 * (its own launch numbers); eps, gate_cap and mlstm_eps are the two layers' common values. A byte outside
 * [0, 512) writes the encoder's NaN outputs and runs neither layer. Added with ABI version 205.
 */
int bp_loc_encdec_step(const bp_loc_layer* enc_layer, const bp_loc_layer* dec_layer, const void* embed,
                       const int64_t* byte, const void* enc_norm, const void* w_patch, const void* w_boundary,
                       void* e_out, void* patch_out, float* boundary_logit, const void* value, const void* w_in,
                       const void* final_norm, const void* lm_head, float* logits, int64_t* out, float eps,
                       float gate_cap, float mlstm_eps, void* workspace, size_t workspace_bytes, void* stream);

/*
 * End of a decode step: out[0] = argmax(logits[0:n]) (torch.argmax order: NaN largest, lowest index on
 * ties), out[1] = sigmoid(*boundary_logit) >= 0.5 (0 when boundary_logit is NULL); out int64.
 * Replaces the argmax and the boundary test of the minimal Bolmo loop (byteprof/optim/bolmo_loop.py:48-53,
 * 182-190).
 */
int bp_decode_finish(const float* logits, int n, const float* boundary_logit, int64_t* out, void* stream);

/*
 * Fused mLSTM recurrence over T positions (exponential gating with the max stabiliser m), one head
 * per group of CTAs, the (C, n, m) state kept on chip across all positions.
 *   c_in [NH, DQ, DV], n_in [NH, DQ], m_in [NH]  fp32, contiguous: the state before position 0
 *   q, k [T, NH, DQ] (row stride str_t_qk), v [T, NH, DV] (str_t_v), elements of `dtype`
 *   i_gate, f_gate [T, NH] pre-activations (str_t_if), elements of `gate_dtype`
 *   h      [T, NH, DV] (str_t_h), `dtype`; NULL = do not compute the outputs
 *   c_out, n_out, m_out  the state after the last applied position; NULL = not written.
 *          c_out may equal c_in (each CTA reads its tile before writing it); n_out / m_out must not
 *          alias n_in / m_in.
 *   n_save, m_save  receive a copy of n_in / m_in (the lazy-commit start copy); NULL = skipped
 *   steps_dev  NULL: apply all T positions. Otherwise a device int64 L: apply positions 0..L
 *          (clamped to T), read on the device so the count can change between graph replays.
 * qk_scale multiplies q (the reference passes DQ^-0.5); eps is added to the denominator.
 * dtype BP_DTYPE_BF16 follows the reference's bf16 casts of the gates, products and C for the
 * output dot product; BP_DTYPE_F32 keeps everything in fp32.
 * Supported: DQ in {64, 128, 256, 512}, DV a multiple of 16; vector strides multiples of 8 elements
 * and 16-byte aligned bases.
 * Replaces multistep_fw_kernel (h only, save n/m) and lazy_commit_kernel (state only, steps_dev),
 * byteprof/optim/mlstm_multistep.py:33-133, and the library step of draft_core.py:114-141 (T = 1).
 */
int bp_mlstm_scan(const float* c_in, const float* n_in, const float* m_in, const void* q, const void* k,
                  const void* v, const void* i_gate, const void* f_gate, void* h, float* c_out, float* n_out,
                  float* m_out, float* n_save, float* m_save, const int64_t* steps_dev, int T, int NH, int DQ,
                  int DV, long long str_t_qk, long long str_t_v, long long str_t_if, long long str_t_h,
                  int dtype, int gate_dtype, float qk_scale, float eps, void* stream);

/*
 * Draft acceptance on the device: out[0:S] <- tok[0:S]; out[smax] <- L, the number of leading
 * drafts ids[1 + j] equal to tok[j] (j < S - 1). ids, tok, out int64.
 * Replaces accept_kernel (byteprof/optim/mlstm_multistep.py:136-146).
 */
int bp_mlstm_accept(const int64_t* ids, const int64_t* tok, int64_t* out, int S, int smax, void* stream);

/*
 * State commit of the drafting loop: cur <- hist[slot] for one layer's state, slot = *slot read on the
 * device (int32 when slot_bytes = 4, int64 when 8), so a captured graph commits whatever length a round
 * accepted. c_hist / n_hist / m_hist hold `slots` consecutive copies of c_count / n_count / m_count fp32
 * values (history slots [slots, 1, NH, DQ, DV], [slots, 1, NH, DQ], [slots, 1, NH, 1]); c_cur / n_cur /
 * m_cur receive slot `slot`. A slot outside [0, slots) fills cur with NaN and reads no history.
 * Replaces commit_state and its commit_kernel (byteprof/optim/draft_core.py:92-111,
 * byteprof/optim/draft_kernels.py:7-18).
 */
int bp_mlstm_commit_state(const float* c_hist, const float* n_hist, const float* m_hist, float* c_cur, float* n_cur,
                          float* m_cur, long long c_count, long long n_count, long long m_count, const void* slot,
                          int slot_bytes, int slots, void* stream);

/*
 * Device error flags raised by the kernels since the last call, then cleared (synchronises the current
 * device). Bit 0: a bounded wait inside a kernel timed out (the kernel stopped early; its output is
 * invalid). No counterpart in the reference, whose kernels have no waits.
 */
int bp_device_errors(unsigned int* flags);

#ifdef __cplusplus
}
#endif

#endif /* BP_KERNELS_H */
