// fitq_nf4_gemv_noalloc: the decode / speculative-verify NF4 GEMV for callers
// that cannot allocate device memory.
//
// Who needs it: a serving runtime or foreign-language host (Go, Java, a C
// inference loop) that drives the decode step through this C ABI but owns no
// CUDA allocator of its own, or that runs under a memory budget where every
// device allocation must be accounted for up front.  Such callers can pass
// inputs and outputs they already hold, but cannot produce the scratch
// workspace fitq_nf4_gemv asks for.  This entry point takes its scratch from a
// fixed array compiled into the library instead, and otherwise IS
// fitq_nf4_gemv: the same argument checks, the same kernel choice for every M
// (decode kernel for M <= 8, tcgen05 skinny GEMM above) and the same
// arithmetic, so its results are bit-identical to fitq_nf4_gemv's.
//
// The scratch is one file-scope __device__ array of kNoAllocScratchBytes
// (8 MiB).  Every GPU that loads the library holds it until the process exits.
// In host code the array's name is only a host-side stand-in; its device
// address is looked up with cudaGetSymbolAddress once per device, with that
// device current, on the first call made on that device.  That first call
// should therefore happen before any stream capture.  All calls share the one
// array and each call overwrites the parts it uses (no kernel of this path
// needs zeroed scratch), so calls that overlap on the GPU -- on two streams,
// or from two host threads -- race on it and must be serialised by the caller.
#include <cstdio>
#include <mutex>

#include "common.cuh"
#include "kernels.cuh"

namespace {

constexpr size_t kNoAllocScratchBytes = FITQ_GEMV_NOALLOC_SCRATCH_BYTES;
constexpr int kMaxDev = 64;

static __device__ __align__(256) uint8_t g_gemv_scratch[kNoAllocScratchBytes];

std::mutex g_mu;
uint8_t* g_scratch_dev[kMaxDev] = {nullptr};

// Errors go to the library's fitq_last_error() text.
int fail(int code, const char* msg) {
  fitq::set_last_error(msg);
  return code;
}

// Device address of the scratch on the current device (set-up on first use).
int scratch_for_current_device(uint8_t** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDev) {
    cudaGetLastError();
    return fail(FITQ_ERR_NO_DEVICE, "nf4_gemv_noalloc: no CUDA device available");
  }
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_scratch_dev[dev] == nullptr) {
    int major = 0;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
    if (major != 10) return fail(FITQ_ERR_NO_DEVICE, "nf4_gemv_noalloc: device is not sm_100");
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_gemv_scratch);
    if (e != cudaSuccess || p == nullptr) {
      char msg[256];
      snprintf(msg, sizeof(msg), "nf4_gemv_noalloc: cudaGetSymbolAddress of the scratch failed (%s)",
               cudaGetErrorString(e));
      cudaGetLastError();
      return fail(FITQ_ERR_CUDA, msg);
    }
    g_scratch_dev[dev] = static_cast<uint8_t*>(p);
  }
  *out = g_scratch_dev[dev];
  return FITQ_OK;
}

}  // namespace

extern "C" {

int fitq_nf4_gemv_noalloc(const fitq_nf4_weight* w, const void* x, int64_t m,
                          const float* lora_a, const float* lora_b, int rank, float scale,
                          const void* bias, void* y, const void* y_add, fitq_stream_t stream) {
  if (!w) return fail(FITQ_ERR_ARG, "nf4_gemv_noalloc: weight descriptor is NULL");
  // The scratch this call would take from a workspace; shapes outside the
  // GEMV's range skip the size check and get their own error below.
  const bool sized = m >= 1 && m <= 64 && w->n_out > 0 && w->k_in > 0 &&
                     w->n_out < (1ll << 31) && w->k_in < (1ll << 31) && rank >= 0 && rank <= 64;
  const size_t need = sized ? fitq_nf4_gemv_workspace(m, w->n_out, w->k_in, rank) : 0;
  if (need > kNoAllocScratchBytes) {
    char msg[256];
    snprintf(msg, sizeof(msg),
             "nf4_gemv_noalloc: this shape needs %zu bytes of scratch, more than the fixed %zu "
             "(use fitq_nf4_gemv with a workspace)",
             need, kNoAllocScratchBytes);
    return fail(FITQ_ERR_WORKSPACE, msg);
  }
  uint8_t* base = nullptr;
  const int rc = scratch_for_current_device(&base);
  if (rc) return rc;
  return fitq::nf4_gemv_on_scratch(w, x, m, lora_a, lora_b, rank, scale, bias, y, y_add, base,
                                   kNoAllocScratchBytes, stream);
}

}  // extern "C"
