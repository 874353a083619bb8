// Forward + backward of the scan in one call, with the chunk-state scratch in a
// file-scope device array instead of caller-provided memory.
//
// Who needs it: callers that cannot allocate device memory themselves or hand us a
// workspace -- e.g. a plugin inside a runtime that owns the whole device memory pool
// (an XLA/JAX process that pre-allocated the GPU, a serving engine with a fixed arena),
// or code that must not call cudaMalloc on its path.  Such a caller still passes the
// inputs and the outputs (o, S_final, the gradient buffers); the chunk-state buffer that the
// two-call API takes from the caller -- sca2_num_chunks(T) slots of K*V fp32 per (b, h): the
// state entering every chunk, the chunk's saved intermediates for the backward and, on the
// explicit-key K = V = 128 path, the backward's workspace -- lives here in
// g_noalloc_chunk_states.
//
// Limits and rules
//   * The array holds SCA2_NOALLOC_SCRATCH_BYTES (16 MiB) on every GPU that loads this
//     library, for the life of the process.  A call needs B*H*NC*K*V*4 bytes
//     (NC = sca2_num_chunks(T)); larger problems are rejected with SCA2_ERR_ARG before
//     anything is launched.
//   * Host code cannot use the array's name as a device address, so the first call on a
//     device (with that device current) looks the address up once with
//     cudaGetSymbolAddress and caches it.  Make that first call before any stream capture.
//   * Every call on a device shares the one array and it keeps the last call's contents.
//     Nothing in it needs clearing: the forward writes every chunk state the backward
//     reads.  Calls whose work overlaps on the GPU (different streams, or host threads
//     racing on one device) race on the array; serialise them.
//   * No cudaMalloc, cudaFree or allocating library routine is called here.
#include <mutex>
#include <string>

#include "common.cuh"

namespace sca2 {
void set_last_error(const std::string& msg);  // capi.cu: the message sca2_last_error() returns
}

namespace {

constexpr size_t kScratchBytes = SCA2_NOALLOC_SCRATCH_BYTES;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) float g_noalloc_chunk_states[kScratchBytes / sizeof(float)];

std::mutex g_mu;
float* g_dev_addr[kMaxDevices] = {};

int noalloc_fail(int code, const std::string& msg) {
  sca2::set_last_error(msg);
  return code;
}

// Device address of the scratch array on the current device (looked up once per device).
int scratch_address(float** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return noalloc_fail(SCA2_ERR_CUDA, std::string("cudaGetDevice: ") + cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) return noalloc_fail(SCA2_ERR_UNSUPPORTED, "device ordinal out of range");
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_dev_addr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_chunk_states);
    if (e != cudaSuccess || !p)
      return noalloc_fail(SCA2_ERR_CUDA, std::string("cudaGetSymbolAddress: ") + cudaGetErrorString(e));
    g_dev_addr[dev] = static_cast<float*>(p);
  }
  *out = g_dev_addr[dev];
  return SCA2_OK;
}

}  // namespace

extern "C" {

int sca2_scan_fwd_bwd_noalloc(const sca2_scan_args* a, sca2_out o, float* S_final, sca2_out dO,
                              const float* dS_final, const sca2_scan_grads* gr, void* stream) {
  if (!a || !gr) return noalloc_fail(SCA2_ERR_ARG, "null argument struct");
  if (a->B < 1 || a->H < 1 || a->K < 1 || a->V < 1 || a->T < 0)
    return noalloc_fail(SCA2_ERR_ARG, "sizes must satisfy B, H, K, V >= 1, T >= 0");
  const int64_t need = (int64_t)a->B * a->H * sca2_num_chunks(a->T) * a->K * a->V * (int64_t)sizeof(float);
  if (need > (int64_t)kScratchBytes)
    return noalloc_fail(SCA2_ERR_ARG, "problem needs " + std::to_string(need) +
                                          " bytes of chunk-state scratch; the no-allocation entry point "
                                          "holds " + std::to_string(kScratchBytes) +
                                          " (use sca2_scan_fwd / sca2_scan_bwd with a caller buffer)");
  float* scratch = nullptr;
  int rc = scratch_address(&scratch);
  if (rc) return rc;
  rc = sca2_scan_fwd(a, o, S_final, scratch, stream);  // writes every chunk state it reads back
  if (rc) return rc;
  return sca2_scan_bwd(a, dO, dS_final, scratch, gr, stream);
}

}  // extern "C"
