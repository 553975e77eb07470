// The per-byte host loop of the batch-1 byte decoder, in C++: per step, the byte goes into a pinned host
// word, one CUDA graph runs the whole byte (its first node copies that word in, its last copies (token,
// boundary flag) out to a pinned pair), the host waits for the stream and reads the pair. A Python loop
// around the same graphs spent ~19 us of host time per byte between the end of one graph and the start of
// the next; here that is a launch and a synchronisation.
//
// Reference: the decode loop of byteprof's minimal Bolmo loop (byteprof/optim/bolmo_loop.py:182-207):
// per byte the encoder graph, the global graph when the previous step flagged a boundary, the decoder
// graph, one synchronisation; the byte decoder here captures the three into one graph per (state parity,
// patch start).
#include <chrono>

#include "bp_common.cuh"

extern "C" int bp_decode_loop(void* const* graph_execs, int64_t* byte_host, const int64_t* out_host,
                              const int64_t* bytes, const int32_t* patches, int n, int64_t first_byte,
                              int32_t first_patch, int parity, int64_t* tokens_out, int32_t* flags_out, void* stream,
                              double* wall_seconds) {
  using namespace bp;
  clear_error();
  if (n < 0) return fail(BP_ERR_INVALID_ARGUMENT, "negative step count %d", n);
  if (graph_execs == nullptr || byte_host == nullptr || out_host == nullptr || tokens_out == nullptr ||
      flags_out == nullptr)
    return fail(BP_ERR_INVALID_ARGUMENT, "a pointer argument is NULL");
  for (int g = 0; g < 4; ++g)
    if (graph_execs[g] == nullptr) return fail(BP_ERR_INVALID_ARGUMENT, "graph %d is NULL", g);
  if (parity != 0 && parity != 1) return fail(BP_ERR_INVALID_ARGUMENT, "parity must be 0 or 1");
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  volatile int64_t* bh = byte_host;
  const volatile int64_t* oh = out_host;
  const auto t0 = std::chrono::steady_clock::now();
  int64_t b = first_byte;
  int32_t patch = first_patch;
  for (int i = 0; i < n; ++i) {
    if (bytes != nullptr) b = bytes[i];
    if (patches != nullptr) patch = patches[i];
    *bh = b;
    const auto exec = static_cast<cudaGraphExec_t>(graph_execs[2 * parity + (patch != 0 ? 1 : 0)]);
    cudaError_t e = cudaGraphLaunch(exec, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return fail(BP_ERR_CUDA, "decode step %d: %s", i, cudaGetErrorString(e));
    tokens_out[i] = oh[0];
    flags_out[i] = static_cast<int32_t>(oh[1]);
    b = tokens_out[i];  // the next step's byte and patch start, unless given
    patch = flags_out[i];
    parity ^= 1;
  }
  if (wall_seconds != nullptr)
    *wall_seconds = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
  return BP_OK;
}
