// fitq_nf4_gemv_noalloc: the decode / speculative-verify NF4 GEMV for callers
// that cannot allocate device memory.
//
// Who needs it: a serving runtime or foreign-language host (Go, Java, a C
// inference loop) that drives the decode step through this C ABI but owns no
// CUDA allocator of its own, or that runs under a memory budget where every
// device allocation must be accounted for up front.  Such callers can pass
// inputs and outputs they already hold, but cannot produce the scratch
// workspace fitq_nf4_gemv asks for.  This entry point takes its scratch from a
// fixed array compiled into the library instead.
//
// The scratch is one file-scope __device__ array of kNoAllocScratchBytes
// (8 MiB).  Every GPU that loads the library holds it until the process exits.
// In host code the array's name is only a host-side stand-in; its device
// address is looked up with cudaGetSymbolAddress once per device, with that
// device current, on the first call made on that device.  That first call
// should therefore happen before any stream capture.  All calls share the one
// array and each call overwrites the parts it uses (nothing has to start at
// zero), so calls that overlap on the GPU -- on two streams, or from two host
// threads -- race on it and must be serialised by the caller.
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
      cudaGetLastError();
      return fail(FITQ_ERR_CUDA, "nf4_gemv_noalloc: cudaGetSymbolAddress of the scratch failed");
    }
    g_scratch_dev[dev] = static_cast<uint8_t*>(p);
  }
  *out = g_scratch_dev[dev];
  return FITQ_OK;
}

inline size_t up256(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }
inline bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

extern "C" {

int fitq_nf4_gemv_noalloc(const fitq_nf4_weight* w, const void* x, int64_t m,
                          const float* lora_a, const float* lora_b, int rank, float scale,
                          const void* bias, void* y, const void* y_add, fitq_stream_t stream) {
  if (!w || !w->packed || !w->quant_map || !x || !y)
    return fail(FITQ_ERR_ARG, "nf4_gemv_noalloc: weight, x and y are required");
  const bool nested = w->absmax_code && w->nested_absmax && w->nested_quant_map;
  if (!nested && !w->absmax_f32)
    return fail(FITQ_ERR_ARG, "nf4_gemv_noalloc: weight has no absmax");
  const int64_t N = w->n_out, K = w->k_in;
  if (m < 1 || m > 64 || N <= 0 || K <= 0 || K % 256 != 0 || N % 64 != 0 || N >= (1ll << 31) ||
      K >= (1ll << 31))
    return fail(FITQ_ERR_SHAPE, "nf4_gemv_noalloc: needs 1 <= M <= 64, K % 256 == 0, N % 64 == 0");
  if (!(rank == 0 || rank == 16 || rank == 32 || rank == 48 || rank == 64))
    return fail(FITQ_ERR_UNSUPPORTED, "nf4_gemv_noalloc: rank must be 0, 16, 32, 48 or 64");
  if (rank > 0 && (!lora_a || !lora_b))
    return fail(FITQ_ERR_ARG, "nf4_gemv_noalloc: lora_a and lora_b are required for rank > 0");
  if (!al16(w->packed) || !al16(x) || !al16(y) || (y_add && !al16(y_add)) || (bias && !al16(bias)))
    return fail(FITQ_ERR_ALIGN, "nf4_gemv_noalloc: pointers must be 16-byte aligned");
  int sms = 0;
  {
    int dev = 0;
    cudaGetDevice(&dev);
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0) {
      cudaGetLastError();
      return fail(FITQ_ERR_NO_DEVICE, "nf4_gemv_noalloc: cannot query the device");
    }
  }
  if (rank > 0 && !al16(lora_b))
    return fail(FITQ_ERR_ALIGN, "nf4_gemv_noalloc: lora_b must be 16-byte aligned");
  // Scratch layout: for the decode kernel (M <= 8): [split-K partials]
  // [T partials]; otherwise [A as bf16 (r x K)][T (M x 64 bf16)]
  // [T partials][split-K partials].
  int slices = 1;
  const bool dec = fitq::gemv_dec_plan(m, N, K, sms, &slices);
  size_t need = 0;
  size_t p_bytes, tp_bytes, t_bytes = 0, a_bytes = 0;
  if (dec) {
    p_bytes = fitq::gemv_dec_needs_partial(slices, rank) ? up256(static_cast<size_t>(slices) * m * N * 4) : 0;
    tp_bytes = rank > 0 ? up256(fitq::lora_t_workspace(m, K, rank)) : 0;
    need += p_bytes + tp_bytes;
  } else {
    a_bytes = rank > 0 ? up256(static_cast<size_t>(rank) * K * 2) : 0;
    t_bytes = rank > 0 ? up256(static_cast<size_t>(m) * 64 * 2) : 0;
    tp_bytes = rank > 0 ? up256(fitq::lora_rowproj_small_workspace(m, K, rank)) : 0;
    p_bytes = up256(fitq::gemv_partial_bytes(m, N, K, sms, nullptr));
    need += a_bytes + t_bytes + tp_bytes + p_bytes;
  }
  if (need > kNoAllocScratchBytes) {
    char msg[256];
    snprintf(msg, sizeof(msg),
             "nf4_gemv_noalloc: this shape needs %zu bytes of scratch, more than the fixed %zu "
             "(use fitq_nf4_gemv with a workspace)",
             need, kNoAllocScratchBytes);
    return fail(FITQ_ERR_WORKSPACE, msg);
  }
  uint8_t* base = nullptr;
  int rc = scratch_for_current_device(&base);
  if (rc) return rc;
  uint8_t* rest = base;

  fitq::Nf4Args a;
  a.packed = w->packed;
  a.absmax_code = nested ? w->absmax_code : nullptr;
  a.nested_absmax = nested ? w->nested_absmax : nullptr;
  a.nested_quant_map = nested ? w->nested_quant_map : nullptr;
  a.absmax_f32 = nested ? nullptr : w->absmax_f32;
  a.quant_map = w->quant_map;
  a.offset = w->offset;
  a.n_out = N;
  a.k_in = K;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (dec) {
    float* partial = p_bytes ? reinterpret_cast<float*>(rest) : nullptr;
    float* t_part = rank > 0 ? reinterpret_cast<float*>(rest + p_bytes) : nullptr;
    fitq::GemvEpilogue ep{y, y_add, bias, lora_b, t_part, fitq::lora_t_groups(K), nullptr,
                          rank, scale, partial};
    if ((rc = fitq::launch_nf4_gemv_dec(a, x, m, ep, st, sms)))
      return fail(rc, "nf4_gemv_noalloc: decode launch failed");
    if (rank > 0 && (rc = fitq::launch_lora_t(x, m, K, lora_a, rank, t_part, st)))
      return fail(rc, "nf4_gemv_noalloc: T = x.A^T launch failed");
    if (partial && (rc = fitq::launch_nf4_gemv_dec_finish(m, N, slices, ep, st, sms)))
      return fail(rc, "nf4_gemv_noalloc: finishing launch failed");
    return FITQ_OK;
  }
  void* a_bf16 = rank > 0 ? rest : nullptr;
  void* t_pad = rank > 0 ? rest + a_bytes : nullptr;
  float* t_part = rank > 0 ? reinterpret_cast<float*>(rest + a_bytes + t_bytes) : nullptr;
  float* partial = reinterpret_cast<float*>(rest + a_bytes + t_bytes + tp_bytes);
  if (rank > 0) {
    if ((rc = fitq::launch_f32_to_bf16(lora_a, static_cast<int64_t>(rank) * K, a_bf16, st)))
      return fail(rc, "nf4_gemv_noalloc: lora_a cast launch failed");
    if ((rc = fitq::launch_lora_rowproj_small(x, K, m, K, a_bf16, rank, t_part, t_pad, nullptr, st)))
      return fail(rc, "nf4_gemv_noalloc: T = x.A^T launch failed");
  }
  int splits = 1;
  if ((rc = fitq::launch_nf4_gemv_core(a, x, m, partial, st, sms, &splits)))
    return fail(rc, "nf4_gemv_noalloc: gemv launch failed");
  if ((rc = fitq::launch_gemv_finish(partial, splits, m, N, t_pad, lora_b, rank, scale, bias, y_add,
                                     y, st, sms)))
    return fail(rc, "nf4_gemv_noalloc: finishing launch failed");
  return FITQ_OK;
}

}  // extern "C"
