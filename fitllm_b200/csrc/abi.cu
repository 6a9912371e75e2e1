// extern "C" entry points of libfitq (declared in include/fitq.h): argument
// checks, workspace carving and kernel sequencing.  No entry point allocates
// device memory; scratch comes from the caller's workspace.
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <atomic>
#include <mutex>
#include <string>
#include <vector>

#include "common.cuh"
#include "kernels.cuh"

// Device status word shared by all kernels of the library (first error wins).
__device__ int g_fitq_status = 0;

namespace {

thread_local std::string g_last_error;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

constexpr int kMaxDevices = 64;

// Number of SMs of the current device; 0 with an error if it is not sm_100.
int current_sms(int* code) {
  static int cache[kMaxDevices] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    cudaGetLastError();
    *code = fail(FITQ_ERR_NO_DEVICE, "no CUDA device available");
    return 0;
  }
  if (cache[dev] == 0) {
    int major = 0, sms = 0;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (major != 10) {
      *code = fail(FITQ_ERR_NO_DEVICE, "device %d is sm_%d0, libfitq is built for sm_100a", dev,
                   major);
      return 0;
    }
    cache[dev] = sms;
  }
  *code = FITQ_OK;
  return cache[dev];
}

// Device address of g_fitq_status on the current device (looked up once per device).
int* status_ptr() {
  static int* cache[kMaxDevices] = {nullptr};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  if (cache[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_fitq_status) != cudaSuccess) {
      cudaGetLastError();
      return nullptr;
    }
    cache[dev] = static_cast<int*>(p);
  }
  return cache[dev];
}

inline bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// A second stream per device for the weight-side launches of one call (the
// NF4 dequant and the LoRA weight padding), which depend on nothing the
// activation-side launches (LoRA casts, row and column projections) produce:
// the call forks it from the caller's stream, runs the two sides
// concurrently and joins it back before the GEMM that needs both.  Fork and
// join are an event record + stream wait each (both allowed during stream
// capture, so a captured call captures the fork); a mutex keeps each
// record/wait pair together when several host threads call in.  When the
// stream cannot be created (or FITQ_SIDE_STREAM=0) the call runs on the
// caller's stream alone, in the same order.
struct SideStream {
  cudaStream_t s = nullptr;
  cudaEvent_t fork = nullptr, join = nullptr;
  bool tried = false;
};
std::mutex g_side_mu;

SideStream* side_stream() {
  static SideStream side[kMaxDevices];
  static const bool off = [] {
    const char* e = getenv("FITQ_SIDE_STREAM");
    return e != nullptr && e[0] == '0';
  }();
  if (off) return nullptr;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    cudaGetLastError();
    return nullptr;
  }
  std::lock_guard<std::mutex> lk(g_side_mu);
  SideStream& ss = side[dev];
  if (!ss.tried) {
    ss.tried = true;
    if (cudaStreamCreateWithFlags(&ss.s, cudaStreamNonBlocking) != cudaSuccess ||
        cudaEventCreateWithFlags(&ss.fork, cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&ss.join, cudaEventDisableTiming) != cudaSuccess) {
      cudaGetLastError();
      ss.s = nullptr;
    }
  }
  return ss.s ? &ss : nullptr;
}

// The stream the weight side runs on: the side stream after a fork from
// `main`, else `main`.
cudaStream_t fork_side(cudaStream_t main, SideStream* ss) {
  if (!ss) return main;
  std::lock_guard<std::mutex> lk(g_side_mu);
  if (cudaEventRecord(ss->fork, main) != cudaSuccess || cudaStreamWaitEvent(ss->s, ss->fork, 0) != cudaSuccess) {
    cudaGetLastError();
    return main;
  }
  return ss->s;
}

// Make `main` wait for everything issued on `side` (no-op when side == main).
int join_side(cudaStream_t main, cudaStream_t side, SideStream* ss) {
  if (side == main) return FITQ_OK;
  std::lock_guard<std::mutex> lk(g_side_mu);
  if (cudaEventRecord(ss->join, side) != cudaSuccess || cudaStreamWaitEvent(main, ss->join, 0) != cudaSuccess)
    return fail(FITQ_ERR_CUDA, "side stream join: %s", cudaGetErrorString(cudaGetLastError()));
  return FITQ_OK;
}



int check_weight(const fitq_nf4_weight* w, fitq::Nf4Args* a) {
  if (!w) return fail(FITQ_ERR_ARG, "weight descriptor is NULL");
  if (!w->packed || !w->quant_map)
    return fail(FITQ_ERR_ARG, "weight: packed and quant_map are required");
  const bool nested = w->absmax_code && w->nested_absmax && w->nested_quant_map;
  if (!nested && !w->absmax_f32)
    return fail(FITQ_ERR_ARG,
                "weight: need absmax_code+nested_absmax+nested_quant_map or absmax_f32");
  if (w->n_out <= 0 || w->k_in <= 0) return fail(FITQ_ERR_SHAPE, "weight: empty shape");
  if (w->k_in % 64 != 0)
    return fail(FITQ_ERR_SHAPE, "weight: K=%lld is not a multiple of the NF4 block (64)",
                (long long)w->k_in);
  if (w->n_out >= (1ll << 31) || w->k_in >= (1ll << 31))
    return fail(FITQ_ERR_SHAPE, "weight: dimension too large");
  if (!al16(w->packed)) return fail(FITQ_ERR_ALIGN, "weight: packed not 16-byte aligned");
  a->packed = w->packed;
  a->absmax_code = nested ? w->absmax_code : nullptr;
  a->nested_absmax = nested ? w->nested_absmax : nullptr;
  a->nested_quant_map = nested ? w->nested_quant_map : nullptr;
  a->absmax_f32 = nested ? nullptr : w->absmax_f32;
  a->quant_map = w->quant_map;
  a->offset = w->offset;
  a->n_out = w->n_out;
  a->k_in = w->k_in;
  return FITQ_OK;
}

// Bump allocator over the caller's workspace (256-byte aligned pieces).
struct Carve {
  uint8_t* base;
  size_t cap;
  size_t used = 0;
  void* take(size_t bytes) {
    size_t off = (used + 255) & ~static_cast<size_t>(255);
    used = off + bytes;
    return base ? base + off : nullptr;
  }
  bool ok() const { return used <= cap; }
};

inline size_t bf16_bytes(int64_t n) { return static_cast<size_t>(n) * 2; }

bool valid_rank(int r) { return r == 0 || r == 16 || r == 32 || r == 48 || r == 64; }

thread_local cudaError_t g_launch_error = cudaSuccess;
thread_local std::string g_launch_detail;

int launch_status(int rc, const char* what) {
  if (rc == FITQ_OK) {
    g_launch_error = cudaSuccess;
    g_launch_detail.clear();
    return FITQ_OK;
  }
  cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) e = g_launch_error;  // a launcher's launch_result() read it already
  g_launch_error = cudaSuccess;
  const std::string detail = g_launch_detail;
  g_launch_detail.clear();
  return fail(rc, "%s: launch failed (%s)%s%s", what, cudaGetErrorString(e), detail.empty() ? "" : "; ",
              detail.c_str());
}

// NF4 dequant fused into the GEMM (gemm_nf4.cu, gemm_nf4_2cta.cu) or the
// materialised dequant + bf16 GEMM, by measured throughput per shape;
// FITQ_NF4_FUSED=1 / 0 in the environment forces one (shapes the fused
// kernels do not take always use the dequant path).
//
// Measured on one B200 (whole call, CUDA-graph replay, L2 flushed): the fused
// kernel wins only where the GEMM's output side is the long one (four times
// the reduction) and the rows are few, so the dequant pass of the 283 MB
// bf16 weight weighs most against the GEMM: at M = 2,048 gate/up forward
// (N 27,648, K 5,120) 448.5 vs 458.8 µs and down_proj dX (output 27,648,
// reduction 5,120) 456.8 vs 471.0 µs; at M = 4,096 and on every other
// Qwen2.5-32B shape the dequant path is faster (up to 1.45x).
bool fused_faster(int64_t m, int64_t n_out, int64_t k_in, int trans) {
  if (m > 2048) return false;
  return trans == 0 ? n_out >= 4 * k_in : k_in >= 4 * n_out;
}

bool use_fused_gemm(int64_t m, int64_t n_out, int64_t k_in, int trans) {
  if (!fitq::gemm_nf4_shape_ok(n_out, k_in, trans)) return false;
  const char* e = getenv("FITQ_NF4_FUSED");
  if (e != nullptr && e[0] == '0') return false;
  if (e != nullptr && e[0] == '1') return true;
  return fused_faster(m, n_out, k_in, trans);
}

// The rank-r projections T = x.A^T and U = dy.B split the reduction over CTAs
// when the rows alone (16 per CTA) would leave most SMs idle.
bool rowproj_split(int64_t m, int sms) { return (m + 15) / 16 < 2 * static_cast<int64_t>(sms); }

// Workspace layout of the forward (shared by the size query and the call).
struct FwdPlan {
  bool fused;      // NF4 decoded inside the GEMM (no wdeq)
  bool gemv;       // M <= 64 skinny path
  bool dec;        // M <= 8 single-launch decode kernel
  bool tc;         // M <= 64 tcgen05 skinny GEMM (weights decoded into TMEM)
  int slices;      // decode K slices
  void* wdeq;      // bf16 [N,K]               (GEMM path)
  void* a_bf16;    // bf16 [r,K]               (rank > 0, not decode)
  void* t_pad;     // bf16 [M,64]              (rank > 0, not decode)
  void* b_pad;     // bf16 [N,64] = s.B        (GEMM path, rank > 0)
  float* partial;  // fp32 [splits,M,N]        (GEMV paths)
  float* t_part;   // fp32 partials of T = x.A^T (GEMV paths, rank > 0)
};

size_t plan_fwd(Carve& c, int64_t m, int64_t n, int64_t k, int rank, int sms, FwdPlan* p) {
  *p = FwdPlan{};
  p->gemv = (m <= 64) && (n % 64 == 0) && (k % 256 == 0);
  p->dec = p->gemv && fitq::gemv_dec_plan(m, n, k, sms, &p->slices);
  p->tc = p->gemv && !p->dec && fitq::gemv_tc_plan(m, n, k, sms, &p->slices);
  if (p->dec || p->tc) {
    if (p->tc || fitq::gemv_dec_needs_partial(p->slices, rank))
      p->partial = static_cast<float*>(c.take(static_cast<size_t>(p->slices * m * n) * sizeof(float)));
    if (rank > 0) p->t_part = static_cast<float*>(c.take(fitq::lora_t_workspace(m, k, rank)));
    return c.used;
  }
  if (rank > 0) {
    p->a_bf16 = c.take(bf16_bytes(static_cast<int64_t>(rank) * k));
    p->t_pad = c.take(bf16_bytes(m * 64));
  }
  if (p->gemv) {
    p->partial = static_cast<float*>(c.take(fitq::gemv_partial_bytes(m, n, k, sms, nullptr)));
    if (rank > 0) p->t_part = static_cast<float*>(c.take(fitq::lora_rowproj_small_workspace(m, k, rank)));
  } else {
    p->fused = use_fused_gemm(m, n, k, 0);
    if (!p->fused) p->wdeq = c.take(bf16_bytes(n * k));
    if (rank > 0) p->b_pad = c.take(bf16_bytes(n * 64));
    if (rank > 0 && rowproj_split(m, sms))
      p->t_part = static_cast<float*>(c.take(fitq::lora_rowproj_small_workspace(m, k, rank)));
  }
  return c.used;
}

struct BwdPlan {
  bool fused;     // dX GEMM decodes W itself (no wt)
  void* wt;       // bf16 [K,N]  transposed dequant
  void* a_bf16;   // bf16 [r,K]  (T recompute)
  void* t_pad;    // bf16 [M,64] (T recompute)
  void* bt_bf16;  // bf16 [r,N]  B^T for U = dy.B
  void* u_pad;    // bf16 [M,64]
  void* at_pad;   // bf16 [K,64] = s.A^T
  float* partial; // colproj scratch
  float* rp_part; // split row projection partials (few rows)
};

size_t plan_bwd(Carve& c, int64_t m, int64_t n, int64_t k, int rank, bool need_dx, bool need_t,
                int sms, BwdPlan* p) {
  *p = BwdPlan{};
  p->fused = need_dx && use_fused_gemm(m, n, k, 1);
  if (need_dx && !p->fused) p->wt = c.take(bf16_bytes(n * k));
  if (rank > 0) {
    if (need_t) {
      p->a_bf16 = c.take(bf16_bytes(static_cast<int64_t>(rank) * k));
      p->t_pad = c.take(bf16_bytes(m * 64));
    }
    p->bt_bf16 = c.take(bf16_bytes(static_cast<int64_t>(rank) * n));
    p->u_pad = c.take(bf16_bytes(m * 64));
    if (need_dx) p->at_pad = c.take(bf16_bytes(k * 64));
    size_t pa = fitq::lora_colproj_workspace(m, k, rank, sms);
    size_t pb = fitq::lora_colproj_workspace(m, n, rank, sms);
    p->partial = static_cast<float*>(c.take(pa > pb ? pa : pb));
    if (rowproj_split(m, sms)) {
      const size_t ra = need_t ? fitq::lora_rowproj_small_workspace(m, k, rank) : 0;
      const size_t rb = fitq::lora_rowproj_small_workspace(m, n, rank);
      p->rp_part = static_cast<float*>(c.take(ra > rb ? ra : rb));
    }
  }
  return c.used;
}

int sms_for_sizing() {
  int code;
  int s = current_sms(&code);
  return s > 0 ? s : 148;
}

}  // namespace

extern "C" {

const char* fitq_version(void) { return "fitq 0.1.0 (sm_100a: tcgen05/TMEM/TMA GEMM, NF4 GEMV)"; }

const char* fitq_last_error(void) { return g_last_error.c_str(); }

int fitq_get_device_status(int reset, fitq_stream_t stream) {
  int code;
  if (current_sms(&code) == 0) return code;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (cudaStreamSynchronize(st) != cudaSuccess)
    return fail(FITQ_ERR_CUDA, "stream sync: %s", cudaGetErrorString(cudaGetLastError()));
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_fitq_status, sizeof(int)) != cudaSuccess)
    return fail(FITQ_ERR_CUDA, "status read: %s", cudaGetErrorString(cudaGetLastError()));
  if (reset) {
    const int zero = 0;
    cudaMemcpyToSymbol(g_fitq_status, &zero, sizeof(int));
  }
  return v;
}

int fitq_selftest_wait_timeout(uint64_t limit_ns, unsigned long long* elapsed_ns,
                               fitq_stream_t stream) {
  int code;
  if (current_sms(&code) == 0) return code;
  if (limit_ns < 1000ull || limit_ns > 1000000000ull)
    return fail(FITQ_ERR_ARG, "selftest_wait_timeout: limit_ns must be in [1e3, 1e9]");
  int* st = status_ptr();
  if (!st) return fail(FITQ_ERR_CUDA, "selftest_wait_timeout: no status word");
  return launch_status(fitq::launch_selftest_wait(limit_ns, elapsed_ns, st,
                                                  static_cast<cudaStream_t>(stream)),
                       "selftest_wait");
}

int fitq_nf4_dequant(const fitq_nf4_weight* w, void* out, int out_dtype, int transpose,
                     fitq_stream_t stream) {
  fitq::Nf4Args a;
  int rc = check_weight(w, &a);
  if (rc) return rc;
  if (!out) return fail(FITQ_ERR_ARG, "dequant: out is NULL");
  if (!al16(out)) return fail(FITQ_ERR_ALIGN, "dequant: out not 16-byte aligned");
  if (out_dtype != FITQ_DTYPE_BF16 && out_dtype != FITQ_DTYPE_F16)
    return fail(FITQ_ERR_ARG, "dequant: unknown out_dtype %d", out_dtype);
  if (transpose && a.n_out % 64 != 0)
    return fail(FITQ_ERR_SHAPE, "dequant: transpose needs N %% 64 == 0 (N=%lld)",
                (long long)a.n_out);
  int sms = current_sms(&rc);
  if (!sms) return rc;
  return launch_status(fitq::launch_nf4_dequant(a, out, out_dtype, transpose,
                                                static_cast<cudaStream_t>(stream), sms),
                       "nf4_dequant");
}

size_t fitq_nf4_quantize_workspace(int64_t n_out, int64_t k_in) {
  Carve c{nullptr, 0};
  const int64_t nb = n_out * k_in / 64;
  c.take(static_cast<size_t>(nb) * sizeof(float));
  c.take(static_cast<size_t>((nb + fitq::kOffsetChunk - 1) / fitq::kOffsetChunk) * sizeof(double));
  return c.used;
}

int fitq_nf4_quantize(const float* w, int64_t n_out, int64_t k_in, const float* quant_map,
                      const float* nested_quant_map, uint8_t* packed, uint8_t* absmax_code,
                      float* nested_absmax, float* offset_out, void* workspace,
                      size_t workspace_bytes, fitq_stream_t stream) {
  if (!w || !quant_map || !nested_quant_map || !packed || !absmax_code || !nested_absmax ||
      !offset_out)
    return fail(FITQ_ERR_ARG, "quantize: NULL argument");
  if (n_out <= 0 || k_in <= 0 || k_in % 64 != 0)
    return fail(FITQ_ERR_SHAPE, "quantize: need K %% 64 == 0 (N=%lld K=%lld)", (long long)n_out,
                (long long)k_in);
  if ((reinterpret_cast<uintptr_t>(w) & 7u) != 0)
    return fail(FITQ_ERR_ALIGN, "quantize: w not 8-byte aligned");
  const size_t need = fitq_nf4_quantize_workspace(n_out, k_in);
  if (!workspace || workspace_bytes < need)
    return fail(FITQ_ERR_WORKSPACE, "quantize: workspace %zu < %zu bytes", workspace_bytes, need);
  int rc;
  int sms = current_sms(&rc);
  if (!sms) return rc;
  Carve c{static_cast<uint8_t*>(workspace), workspace_bytes};
  const int64_t nb = n_out * k_in / 64;
  float* absmax = static_cast<float*>(c.take(static_cast<size_t>(nb) * sizeof(float)));
  double* partial = static_cast<double*>(
      c.take(static_cast<size_t>((nb + fitq::kOffsetChunk - 1) / fitq::kOffsetChunk) *
             sizeof(double)));
  return launch_status(fitq::launch_nf4_quantize(w, n_out * k_in, quant_map, nested_quant_map,
                                                 packed, absmax_code, nested_absmax, offset_out,
                                                 absmax, partial,
                                                 static_cast<cudaStream_t>(stream), sms),
                       "nf4_quantize");
}

size_t fitq_qlora_fwd_workspace(int64_t m, int64_t n_out, int64_t k_in, int rank) {
  Carve c{nullptr, 0};
  FwdPlan p;
  return plan_fwd(c, m, n_out, k_in, rank, sms_for_sizing(), &p);
}

}  // extern "C"

static int qlora_fwd_impl(const fitq_nf4_weight* w, const void* x, int64_t m, const float* lora_a,
                          const float* lora_b, int rank, float scale, const void* bias, void* y,
                          const void* y_add,
                          void* t_out, void* workspace, size_t workspace_bytes,
                          fitq_stream_t stream, int force_gemv) {
  fitq::Nf4Args a;
  int rc = check_weight(w, &a);
  if (rc) return rc;
  if (!x || !y) return fail(FITQ_ERR_ARG, "qlora_fwd: x and y are required");
  if (m <= 0 || m >= (1ll << 31)) return fail(FITQ_ERR_SHAPE, "qlora_fwd: bad M=%lld", (long long)m);
  if (!valid_rank(rank)) return fail(FITQ_ERR_UNSUPPORTED, "qlora_fwd: rank %d not in {0,16,32,48,64}", rank);
  if (rank > 0 && (!lora_a || !lora_b)) return fail(FITQ_ERR_ARG, "qlora_fwd: lora_a/lora_b required for rank > 0");
  if (rank > 0 && (!al16(lora_a) || !al16(lora_b)))
    return fail(FITQ_ERR_ALIGN, "qlora_fwd: lora_a / lora_b must be 16-byte aligned");
  if (a.n_out % 16 != 0) return fail(FITQ_ERR_SHAPE, "qlora_fwd: N=%lld not a multiple of 16", (long long)a.n_out);
  if (!al16(x) || !al16(y) || (y_add && !al16(y_add)) || (t_out && !al16(t_out)) ||
      (bias && !al16(bias)))
    return fail(FITQ_ERR_ALIGN, "qlora_fwd: x/y/bias/y_add/t_out must be 16-byte aligned");
  int sms = current_sms(&rc);
  if (!sms) return rc;
  const int64_t N = a.n_out, K = a.k_in;
  Carve probe{nullptr, 0};
  FwdPlan p;
  const size_t need = plan_fwd(probe, m, N, K, rank, sms, &p);
  if (force_gemv && !p.gemv)
    return fail(FITQ_ERR_SHAPE,
                "nf4_gemv: needs M <= 64, N %% 64 == 0 and K %% 256 == 0 (M=%lld N=%lld K=%lld)",
                (long long)m, (long long)N, (long long)K);
  if (workspace_bytes < need || (need > 0 && !workspace))
    return fail(FITQ_ERR_WORKSPACE, "qlora_fwd: workspace %zu < %zu bytes", workspace_bytes, need);
  Carve c{static_cast<uint8_t*>(workspace), workspace_bytes};
  plan_fwd(c, m, N, K, rank, sms, &p);
  if (!c.ok())  // the size query and the call carve the same plan: never past the end
    return fail(FITQ_ERR_WORKSPACE, "qlora_fwd: plan of %zu bytes exceeds the workspace", c.used);
  cudaStream_t st = static_cast<cudaStream_t>(stream);

  if (p.dec || p.tc) {
    // GEMV, then T (overlapping the weight stream), then the finishing sum
    fitq::GemvEpilogue ep{y, y_add, bias, lora_b, p.t_part, fitq::lora_t_groups(K), t_out,
                          rank, scale, p.partial};
    rc = p.dec ? fitq::launch_nf4_gemv_dec(a, x, m, ep, st, sms)
               : fitq::launch_nf4_gemv_tc(a, x, m, p.partial, status_ptr(), st, sms);
    if (rc) return launch_status(rc, p.dec ? "nf4_gemv decode" : "nf4_gemv tcgen05");
    if (rank > 0) {
      rc = fitq::launch_lora_t(x, m, K, lora_a, rank, p.t_part, st);
      if (rc) return launch_status(rc, "lora T = x.A^T");
    }
    if (p.partial)
      return launch_status(fitq::launch_nf4_gemv_dec_finish(m, N, p.slices, ep, st, sms),
                           "nf4_gemv decode finish");
    return FITQ_OK;
  }
  // GEMM path: the weight side (s.B padding, NF4 dequant) on the side stream
  // while T = x.A^T runs on the caller's stream; joined before the GEMM.
  SideStream* ss = (!p.gemv && !p.fused) ? side_stream() : nullptr;
  cudaStream_t wst = fork_side(st, ss);
  int wrc = FITQ_OK;
  const char* wwhat = "";
  if (!p.gemv) {
    if (rank > 0 && (wrc = fitq::launch_pad_lora_weight(lora_b, N, rank, scale, 0, p.b_pad, wst)))
      wwhat = "lora B pad";
    if (!wrc && !p.fused && (wrc = fitq::launch_nf4_dequant(a, p.wdeq, FITQ_DTYPE_BF16, 0, wst, sms)))
      wwhat = "nf4_dequant";
  }
  if (rank > 0) {
    rc = fitq::launch_f32_to_bf16(lora_a, static_cast<int64_t>(rank) * K, p.a_bf16, st);
    if (!rc)
      rc = p.t_part ? fitq::launch_lora_rowproj_small(x, K, m, K, p.a_bf16, rank, p.t_part, p.t_pad,
                                                      t_out, st)
                    : fitq::launch_lora_rowproj(x, K, m, K, p.a_bf16, rank, p.t_pad, t_out, st, sms);
  }
  const int jrc = join_side(st, wst, ss);
  if (wrc) return launch_status(wrc, wwhat);
  if (rc) return launch_status(rc, "lora T = x.A^T");
  if (jrc) return jrc;
  if (p.gemv) {
    int splits = 1;
    rc = fitq::launch_nf4_gemv_core(a, x, m, p.partial, st, sms, &splits);
    if (rc) return launch_status(rc, "nf4_gemv");
    rc = fitq::launch_gemv_finish(p.partial, splits, m, N, p.t_pad, lora_b, rank, scale, bias,
                                  y_add, y, st, sms);
    return launch_status(rc, "nf4_gemv finish");
  }
  if (p.fused) {
    fitq::Nf4GemmArgs g{};
    g.w = a; g.trans = 0;
    g.a = x; g.lda = K;
    g.pa = p.t_pad; g.pb = p.b_pad;
    g.c = y; g.ldc = N;
    g.c_add = y_add; g.ldc_add = N;
    g.bias = bias;
    g.m = m;
    g.lora_k = rank;
    g.status = status_ptr();
    return launch_status(fitq::launch_gemm_nf4(g, st, sms), "tcgen05 nf4 gemm");
  }
  fitq::GemmArgs g{};
  g.a = x; g.lda = K;
  g.b = p.wdeq; g.ldb = K;
  g.pa = p.t_pad; g.pb = p.b_pad;
  g.c = y; g.ldc = N;
  g.c_add = y_add; g.ldc_add = N;
  g.bias = bias;
  g.m = m; g.n = N; g.k = K;
  g.lora_k = rank;
  g.status = status_ptr();
  return launch_status(fitq::launch_gemm(g, st, sms), "tcgen05 gemm");
}

namespace fitq {
// fitq_nf4_gemv over a caller-chosen scratch (the no-allocation entry point
// passes its fixed device array): same checks, plan and launches.
int nf4_gemv_on_scratch(const fitq_nf4_weight* w, const void* x, int64_t m, const float* lora_a,
                        const float* lora_b, int rank, float scale, const void* bias, void* y,
                        const void* y_add, void* scratch, size_t scratch_bytes,
                        fitq_stream_t stream) {
  return qlora_fwd_impl(w, x, m, lora_a, lora_b, rank, scale, bias, y, y_add, nullptr, scratch,
                        scratch_bytes, stream, 1);
}
}  // namespace fitq

extern "C" {

int fitq_qlora_fwd(const fitq_nf4_weight* w, const void* x, int64_t m, const float* lora_a,
                   const float* lora_b, int rank, float scale, const void* bias, void* y,
                   const void* y_add, void* t_out, void* workspace, size_t workspace_bytes,
                   fitq_stream_t stream) {
  return qlora_fwd_impl(w, x, m, lora_a, lora_b, rank, scale, bias, y, y_add, t_out, workspace,
                        workspace_bytes, stream, 0);
}

size_t fitq_nf4_gemv_workspace(int64_t m, int64_t n_out, int64_t k_in, int rank) {
  return fitq_qlora_fwd_workspace(m, n_out, k_in, rank);
}

int fitq_nf4_gemv(const fitq_nf4_weight* w, const void* x, int64_t m, const float* lora_a,
                  const float* lora_b, int rank, float scale, const void* bias, void* y,
                  const void* y_add, void* workspace, size_t workspace_bytes,
                  fitq_stream_t stream) {
  return qlora_fwd_impl(w, x, m, lora_a, lora_b, rank, scale, bias, y, y_add, nullptr, workspace,
                        workspace_bytes, stream, 1);
}

// Grouped GEMV: the single tcgen05 launch applies when every job shares K and
// the scale format, N % 128 == 0 and the tcgen05 plan takes M for the summed N.
static bool grouped_tc(const fitq_gemv_job* jobs, int count, int64_t m, int sms, int* slices) {
  if (count < 1 || count > 3) return false;
  const fitq_nf4_weight* w0 = jobs[0].w;
  if (!w0) return false;
  const bool nested = w0->absmax_f32 == nullptr;
  int64_t n_total = 0;
  for (int g = 0; g < count; ++g) {
    const fitq_nf4_weight* w = jobs[g].w;
    if (!w || w->k_in != w0->k_in || (w->absmax_f32 == nullptr) != nested || w->n_out % 128 != 0)
      return false;
    n_total += w->n_out;
  }
  return fitq::gemv_tc_plan(m, n_total, w0->k_in, sms, slices);
}

// Grouped decode launch (M <= 8): two or three jobs sharing K and the scale
// format, N % 64 == 0 each, and a decode plan for the summed N.
static bool grouped_dec(const fitq_gemv_job* jobs, int count, int64_t m, int sms, int* slices) {
  if (count < 2 || count > 3) return false;
  const fitq_nf4_weight* w0 = jobs[0].w;
  if (!w0) return false;
  const bool nested = w0->absmax_f32 == nullptr;
  int64_t n_total = 0;
  for (int g = 0; g < count; ++g) {
    const fitq_nf4_weight* w = jobs[g].w;
    if (!w || w->k_in != w0->k_in || (w->absmax_f32 == nullptr) != nested || w->n_out % 64 != 0)
      return false;
    n_total += w->n_out;
  }
  return fitq::gemv_dec_plan(m, n_total, w0->k_in, sms, slices);
}

static size_t grouped_bytes(const fitq_gemv_job* jobs, int count, int64_t m, int slices) {
  Carve c{nullptr, 0};
  for (int g = 0; g < count; ++g) {
    c.take(static_cast<size_t>(slices) * m * jobs[g].w->n_out * sizeof(float));
    if (jobs[g].rank > 0) c.take(fitq::lora_t_workspace(m, jobs[g].w->k_in, jobs[g].rank));
  }
  return c.used;
}

// Bytes of the fallback of the SwiGLU entry: gate and up outputs (bf16) ahead
// of the per-projection GEMV workspace.
static size_t swiglu_scratch_bytes(const fitq_gemv_job* jobs, int64_t m) {
  return 2 * ((static_cast<size_t>(m) * jobs[0].w->n_out * 2 + 255) / 256 * 256);
}

static size_t grouped_workspace(const fitq_gemv_job* jobs, int count, int64_t m, bool swiglu) {
  if (!jobs || count < 1 || count > 3) return 0;
  for (int g = 0; g < count; ++g)
    if (!jobs[g].w) return 0;
  const int sms = sms_for_sizing();
  int slices = 0;
  if (grouped_tc(jobs, count, m, sms, &slices) || grouped_dec(jobs, count, m, sms, &slices))
    return grouped_bytes(jobs, count, m, slices);
  size_t need = 0;
  for (int g = 0; g < count; ++g) {
    const size_t b = fitq_nf4_gemv_workspace(m, jobs[g].w->n_out, jobs[g].w->k_in, jobs[g].rank);
    need = b > need ? b : need;
  }
  return need + (swiglu ? swiglu_scratch_bytes(jobs, m) : 0);
}

size_t fitq_nf4_gemv_grouped_workspace(const fitq_gemv_job* jobs, int count, int64_t m) {
  return grouped_workspace(jobs, count, m, false);
}

size_t fitq_nf4_gemv_swiglu_workspace(const fitq_gemv_job* jobs, int64_t m) {
  return grouped_workspace(jobs, 2, m, true);
}

// One grouped launch of 1-3 projections of x; with act set (the SwiGLU entry)
// the two results are combined in the finishing pass and only act is stored.
static int grouped_impl(const fitq_gemv_job* jobs, int count, const void* x, int64_t m, void* act,
                        void* workspace, size_t workspace_bytes, fitq_stream_t stream) {
  const char* what = act ? "nf4_gemv_swiglu" : "nf4_gemv_grouped";
  int rc;
  const int sms = current_sms(&rc);
  if (!sms) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int slices = 0;
  const bool tc = grouped_tc(jobs, count, m, sms, &slices);
  if (!tc && !grouped_dec(jobs, count, m, sms, &slices)) {
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    size_t left = workspace_bytes;
    void* y[3] = {nullptr, nullptr, nullptr};
    if (act) {  // gate and up into the workspace, then the elementwise kernel
      const size_t scratch = swiglu_scratch_bytes(jobs, m);
      if (!ws || left < scratch)
        return fail(FITQ_ERR_WORKSPACE, "%s: workspace %zu < %zu bytes", what, left, scratch);
      y[0] = ws;
      y[1] = ws + scratch / 2;
      ws += scratch;
      left -= scratch;
    }
    for (int g = 0; g < count; ++g) {
      const fitq_gemv_job& j = jobs[g];
      rc = fitq_nf4_gemv(j.w, x, m, j.lora_a, j.lora_b, j.rank, j.scale, j.bias, act ? y[g] : j.y,
                         j.y_add, ws, left, stream);
      if (rc) return rc;
    }
    if (act)
      return launch_status(fitq::launch_swiglu_fwd(y[0], y[1], act, m * jobs[0].w->n_out, st, sms),
                           "swiglu_fwd");
    return FITQ_OK;
  }
  // the checks of fitq_nf4_gemv, per job
  fitq::Nf4Args a[3];
  for (int g = 0; g < count; ++g) {
    const fitq_gemv_job& j = jobs[g];
    if ((rc = check_weight(j.w, &a[g]))) return rc;
    if (!x || (!act && !j.y)) return fail(FITQ_ERR_ARG, "%s: x and y are required", what);
    if (!valid_rank(j.rank)) return fail(FITQ_ERR_UNSUPPORTED, "%s: rank %d", what, j.rank);
    if (j.rank > 0 && (!j.lora_a || !j.lora_b || !al16(j.lora_a) || !al16(j.lora_b)))
      return fail(FITQ_ERR_ALIGN, "%s: lora_a / lora_b required, 16-byte aligned", what);
    if (!al16(x) || (j.y && !al16(j.y)) || (j.y_add && !al16(j.y_add)) || (j.bias && !al16(j.bias)))
      return fail(FITQ_ERR_ALIGN, "%s: x/y/bias/y_add must be 16-byte aligned", what);
  }
  const size_t need = grouped_bytes(jobs, count, m, slices);
  if (workspace_bytes < need || !workspace)
    return fail(FITQ_ERR_WORKSPACE, "%s: workspace %zu < %zu bytes", what, workspace_bytes, need);
  Carve c{static_cast<uint8_t*>(workspace), workspace_bytes};
  float* partial[3] = {nullptr, nullptr, nullptr};
  float* t_part[3] = {nullptr, nullptr, nullptr};
  for (int g = 0; g < count; ++g) {
    partial[g] = static_cast<float*>(c.take(static_cast<size_t>(slices) * m * a[g].n_out * sizeof(float)));
    if (jobs[g].rank > 0)
      t_part[g] = static_cast<float*>(c.take(fitq::lora_t_workspace(m, a[g].k_in, jobs[g].rank)));
  }
  if (!c.ok()) return fail(FITQ_ERR_WORKSPACE, "%s: plan of %zu bytes exceeds the workspace", what, c.used);
  const int64_t K = a[0].k_in;
  rc = tc ? fitq::launch_nf4_gemv_tc_grouped(a, count, x, m, partial, status_ptr(), st, sms)
          : fitq::launch_nf4_gemv_dec_grouped(a, count, x, m, partial, status_ptr(), st, sms);
  if (rc) return launch_status(rc, tc ? "nf4_gemv_grouped tcgen05" : "nf4_gemv_grouped decode");
  fitq::GemvEpilogue ep[3];
  int64_t n_out[3];
  const float* t_a[3];
  int t_r[3];
  float* t_out[3];
  int t_jobs = 0;
  for (int g = 0; g < count; ++g) {
    const fitq_gemv_job& j = jobs[g];
    if (j.rank > 0) {  // every job's T partials in one launch
      t_a[t_jobs] = j.lora_a;
      t_r[t_jobs] = j.rank;
      t_out[t_jobs] = t_part[g];
      ++t_jobs;
    }
    ep[g] = fitq::GemvEpilogue{j.y, j.y_add, j.bias, j.lora_b, t_part[g], fitq::lora_t_groups(K), nullptr,
                               j.rank, j.scale, partial[g]};
    n_out[g] = a[g].n_out;
  }
  if (t_jobs > 0 && (rc = fitq::launch_lora_t_multi(x, m, K, t_a, t_r, t_out, t_jobs, st)))
    return launch_status(rc, "lora T = x.A^T");
  return launch_status(fitq::launch_nf4_gemv_group_finish(m, n_out, count, slices, ep, act, st),
                       "nf4_gemv_grouped finish");
}

int fitq_nf4_gemv_grouped(const fitq_gemv_job* jobs, int count, const void* x, int64_t m,
                          void* workspace, size_t workspace_bytes, fitq_stream_t stream) {
  if (!jobs || count < 1 || count > 3) return fail(FITQ_ERR_ARG, "nf4_gemv_grouped: 1 to 3 jobs");
  return grouped_impl(jobs, count, x, m, nullptr, workspace, workspace_bytes, stream);
}

int fitq_nf4_gemv_swiglu(const fitq_gemv_job* jobs, const void* x, int64_t m, void* act,
                         void* workspace, size_t workspace_bytes, fitq_stream_t stream) {
  if (!jobs || !jobs[0].w || !jobs[1].w || !act)
    return fail(FITQ_ERR_ARG, "nf4_gemv_swiglu: gate, up and act are required");
  if (jobs[0].w->n_out != jobs[1].w->n_out || jobs[0].w->k_in != jobs[1].w->k_in)
    return fail(FITQ_ERR_SHAPE, "nf4_gemv_swiglu: gate and up must have the same shape");
  if (jobs[0].rank != 0 || jobs[1].rank != 0)
    return fail(FITQ_ERR_UNSUPPORTED, "nf4_gemv_swiglu: gate/up with LoRA are not fused");
  if (m <= 0 || (m * jobs[0].w->n_out) % 8 != 0)
    return fail(FITQ_ERR_SHAPE, "nf4_gemv_swiglu: need m * n_out %% 8 == 0");
  if (!al16(act)) return fail(FITQ_ERR_ALIGN, "nf4_gemv_swiglu: act must be 16-byte aligned");
  return grouped_impl(jobs, 2, x, m, act, workspace, workspace_bytes, stream);
}

size_t fitq_qlora_bwd_workspace(int64_t m, int64_t n_out, int64_t k_in, int rank) {
  Carve c{nullptr, 0};
  BwdPlan p;
  return plan_bwd(c, m, n_out, k_in, rank, true, true, sms_for_sizing(), &p);
}

static int lora_bwd_side(const void* x, const void* dy, int64_t m, int64_t N, int64_t K,
                         const float* lora_a, const float* lora_b, int rank, float scale,
                         const void* t_saved, bool need_t, float* grad_a, float* grad_b,
                         int grad_accumulate, const BwdPlan& p, cudaStream_t st, int sms);

int fitq_qlora_bwd(const fitq_nf4_weight* w, const void* x, const void* dy, int64_t m,
                   const float* lora_a, const float* lora_b, int rank, float scale,
                   const void* t_saved, void* dx, int dx_accumulate, float* grad_a,
                   float* grad_b, int grad_accumulate, void* workspace, size_t workspace_bytes,
                   fitq_stream_t stream) {
  fitq::Nf4Args a;
  int rc = check_weight(w, &a);
  if (rc) return rc;
  if (!dy) return fail(FITQ_ERR_ARG, "qlora_bwd: dy is required");
  if (m <= 0 || m >= (1ll << 31)) return fail(FITQ_ERR_SHAPE, "qlora_bwd: bad M=%lld", (long long)m);
  if (!valid_rank(rank)) return fail(FITQ_ERR_UNSUPPORTED, "qlora_bwd: rank %d not in {0,16,32,48,64}", rank);
  if (rank > 0 && (!lora_a || !lora_b || !grad_a || !grad_b || !x))
    return fail(FITQ_ERR_ARG, "qlora_bwd: x, lora_a/b and grad_a/b are required for rank > 0");
  const int64_t N = a.n_out, K = a.k_in;
  if (N % 64 != 0) return fail(FITQ_ERR_SHAPE, "qlora_bwd: N=%lld not a multiple of 64", (long long)N);
  if (!al16(dy) || (x && !al16(x)) || (dx && !al16(dx)) || (t_saved && !al16(t_saved)))
    return fail(FITQ_ERR_ALIGN, "qlora_bwd: x/dy/dx/t_saved must be 16-byte aligned");
  int sms = current_sms(&rc);
  if (!sms) return rc;
  const bool need_dx = dx != nullptr;
  const bool need_t = rank > 0 && t_saved == nullptr;
  Carve probe{nullptr, 0};
  BwdPlan p;
  const size_t need = plan_bwd(probe, m, N, K, rank, need_dx, need_t, sms, &p);
  if (workspace_bytes < need || (need > 0 && !workspace))
    return fail(FITQ_ERR_WORKSPACE, "qlora_bwd: workspace %zu < %zu bytes", workspace_bytes, need);
  Carve c{static_cast<uint8_t*>(workspace), workspace_bytes};
  plan_bwd(c, m, N, K, rank, need_dx, need_t, sms, &p);
  if (!c.ok())
    return fail(FITQ_ERR_WORKSPACE, "qlora_bwd: plan of %zu bytes exceeds the workspace", c.used);
  cudaStream_t st = static_cast<cudaStream_t>(stream);

  // The weight side of dX (s.A^T padding, transposed NF4 dequant) on the side
  // stream while the LoRA projections run on the caller's stream.
  SideStream* ss = (need_dx && !p.fused) ? side_stream() : nullptr;
  cudaStream_t wst = fork_side(st, ss);
  int wrc = FITQ_OK;
  const char* wwhat = "";
  if (need_dx) {
    if (rank > 0 && (wrc = fitq::launch_pad_lora_weight(lora_a, K, rank, scale, 1, p.at_pad, wst)))
      wwhat = "lora A^T pad";
    if (!wrc && !p.fused && (wrc = fitq::launch_nf4_dequant(a, p.wt, FITQ_DTYPE_BF16, 1, wst, sms)))
      wwhat = "nf4_dequant (transposed)";
  }
  rc = lora_bwd_side(x, dy, m, N, K, lora_a, lora_b, rank, scale, t_saved, need_t, grad_a, grad_b,
                     grad_accumulate, p, st, sms);
  const int jrc = join_side(st, wst, ss);
  if (wrc) return launch_status(wrc, wwhat);
  if (rc) return rc;
  if (jrc) return jrc;
  if (!need_dx) return FITQ_OK;
  // dx[M, K] = dy[M, N].W[N, K] + U.(s.A), W decoded inside the GEMM, or
  // W^T materialised [K, N] bf16 first (bit-exact dequant either way).
  if (p.fused) {
    fitq::Nf4GemmArgs g{};
    g.w = a; g.trans = 1;
    g.a = dy; g.lda = N;
    g.pa = p.u_pad; g.pb = p.at_pad;
    g.c = dx; g.ldc = K;
    g.c_add = dx_accumulate ? dx : nullptr; g.ldc_add = K;
    g.m = m;
    g.lora_k = rank;
    g.status = status_ptr();
    return launch_status(fitq::launch_gemm_nf4(g, st, sms), "tcgen05 nf4 gemm (dx)");
  }
  fitq::GemmArgs g{};
  g.a = dy; g.lda = N;
  g.b = p.wt; g.ldb = N;
  g.pa = p.u_pad; g.pb = p.at_pad;
  g.c = dx; g.ldc = K;
  g.c_add = dx_accumulate ? dx : nullptr; g.ldc_add = K;
  g.m = m; g.n = K; g.k = N;
  g.lora_k = rank;
  g.status = status_ptr();
  return launch_status(fitq::launch_gemm(g, st, sms), "tcgen05 gemm (dx)");
}

// LoRA part of the backward on stream st: T recompute (when not saved),
// U = dy.B, dB = s.dy^T.T, dA = s.U^T.x.
static int lora_bwd_side(const void* x, const void* dy, int64_t m, int64_t N, int64_t K,
                         const float* lora_a, const float* lora_b, int rank, float scale,
                         const void* t_saved, bool need_t, float* grad_a, float* grad_b,
                         int grad_accumulate, const BwdPlan& p, cudaStream_t st, int sms) {
  int rc = FITQ_OK;
  const void* t_ptr = t_saved;
  int64_t t_ld = rank;
  if (rank > 0) {
    if (need_t) {
      rc = fitq::launch_f32_to_bf16(lora_a, static_cast<int64_t>(rank) * K, p.a_bf16, st);
      if (rc) return launch_status(rc, "lora_a cast");
      rc = p.rp_part ? fitq::launch_lora_rowproj_small(x, K, m, K, p.a_bf16, rank, p.rp_part,
                                                       p.t_pad, nullptr, st)
                     : fitq::launch_lora_rowproj(x, K, m, K, p.a_bf16, rank, p.t_pad, nullptr, st, sms);
      if (rc) return launch_status(rc, "lora T recompute");
      t_ptr = p.t_pad;
      t_ld = 64;
    }
    // U = dy.B, with B^T cast to bf16 [r, N]
    rc = fitq::launch_f32_to_bf16_t(lora_b, N, rank, p.bt_bf16, st);
    if (rc) return launch_status(rc, "lora_b cast");
    rc = p.rp_part ? fitq::launch_lora_rowproj_small(dy, N, m, N, p.bt_bf16, rank, p.rp_part,
                                                     p.u_pad, nullptr, st)
                   : fitq::launch_lora_rowproj(dy, N, m, N, p.bt_bf16, rank, p.u_pad, nullptr, st, sms);
    if (rc) return launch_status(rc, "lora U = dy.B");
    // dB[N, r] = s.dy^T.T ; dA[r, K] = s.U^T.x
    rc = fitq::launch_lora_colproj(t_ptr, t_ld, dy, N, m, N, rank, scale, grad_b, 1,
                                   grad_accumulate, p.partial, st, sms);
    if (rc) return launch_status(rc, "lora dB");
    rc = fitq::launch_lora_colproj(p.u_pad, 64, x, K, m, K, rank, scale, grad_a, 0,
                                   grad_accumulate, p.partial, st, sms);
    if (rc) return launch_status(rc, "lora dA");
  }
  return FITQ_OK;
}

size_t fitq_nf4_gateup_swiglu_workspace(int64_t m, int64_t n_out, int64_t k_in) {
  (void)m;
  Carve c{nullptr, 0};
  c.take(bf16_bytes(n_out * k_in));
  c.take(bf16_bytes(n_out * k_in));
  return c.used;
}

int fitq_nf4_gateup_swiglu(const fitq_nf4_weight* w_gate, const fitq_nf4_weight* w_up, const void* x,
                           int64_t m, void* act, void* gate_out, void* up_out, void* workspace,
                           size_t workspace_bytes, fitq_stream_t stream) {
  fitq::Nf4Args g, u;
  int rc = check_weight(w_gate, &g);
  if (rc) return rc;
  if ((rc = check_weight(w_up, &u))) return rc;
  if (g.n_out != u.n_out || g.k_in != u.k_in)
    return fail(FITQ_ERR_SHAPE, "gateup_swiglu: gate and up must have the same shape");
  if (!x || !act) return fail(FITQ_ERR_ARG, "gateup_swiglu: x and act are required");
  if (m <= 0 || m >= (1ll << 31)) return fail(FITQ_ERR_SHAPE, "gateup_swiglu: bad M=%lld", (long long)m);
  const int64_t N = g.n_out, K = g.k_in;
  if (N % 128 != 0)
    return fail(FITQ_ERR_SHAPE, "gateup_swiglu: N=%lld not a multiple of 128", (long long)N);
  if (!al16(x) || !al16(act) || (gate_out && !al16(gate_out)) || (up_out && !al16(up_out)))
    return fail(FITQ_ERR_ALIGN, "gateup_swiglu: x/act/gate_out/up_out must be 16-byte aligned");
  const size_t need = fitq_nf4_gateup_swiglu_workspace(m, N, K);
  if (!workspace || workspace_bytes < need)
    return fail(FITQ_ERR_WORKSPACE, "gateup_swiglu: workspace %zu < %zu bytes", workspace_bytes, need);
  int sms = current_sms(&rc);
  if (!sms) return rc;
  Carve c{static_cast<uint8_t*>(workspace), workspace_bytes};
  void* wg = c.take(bf16_bytes(N * K));
  void* wu = c.take(bf16_bytes(N * K));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if ((rc = fitq::launch_nf4_dequant(g, wg, FITQ_DTYPE_BF16, 0, st, sms)))
    return launch_status(rc, "nf4_dequant (gate)");
  if ((rc = fitq::launch_nf4_dequant(u, wu, FITQ_DTYPE_BF16, 0, st, sms)))
    return launch_status(rc, "nf4_dequant (up)");
  fitq::GemmArgs a{};
  a.a = x; a.lda = K;
  a.b = wg; a.b2 = wu; a.ldb = K;
  a.c = act; a.ldc = N;
  a.m = m; a.n = N; a.k = K;
  a.epi = fitq::GEMM_EPI_SWIGLU;
  a.aux0 = gate_out; a.aux1 = up_out;
  a.status = status_ptr();
  return launch_status(fitq::launch_gemm(a, st, sms), "tcgen05 gemm (gate/up + SwiGLU)");
}

int fitq_lora_merge(void* w, int w_dtype, int64_t n_out, int64_t k_in, const float* lora_a,
                    const float* lora_b, int rank, float scale, fitq_stream_t stream) {
  if (!w || !lora_a || !lora_b) return fail(FITQ_ERR_ARG, "lora_merge: w, lora_a and lora_b are required");
  if (w_dtype != FITQ_DTYPE_BF16 && w_dtype != FITQ_DTYPE_F16 && w_dtype != FITQ_DTYPE_F32)
    return fail(FITQ_ERR_ARG, "lora_merge: unknown w_dtype %d", w_dtype);
  if (n_out <= 0 || k_in <= 0 || (k_in & 1) || n_out >= (1ll << 31) || k_in >= (1ll << 31) ||
      (n_out + 15) / 16 > 65535)
    return fail(FITQ_ERR_SHAPE, "lora_merge: bad shape N=%lld K=%lld (K even)", (long long)n_out,
                (long long)k_in);
  if (rank < 1 || rank > 256) return fail(FITQ_ERR_SHAPE, "lora_merge: rank %d not in 1..256", rank);
  if ((reinterpret_cast<uintptr_t>(w) & (w_dtype == FITQ_DTYPE_F32 ? 7u : 3u)) ||
      (reinterpret_cast<uintptr_t>(lora_a) & 7u) ||
      (reinterpret_cast<uintptr_t>(lora_b) & 3u))
    return fail(FITQ_ERR_ALIGN, "lora_merge: w 4-byte (fp32: 8-byte), lora_a 8-byte, lora_b 4-byte alignment");
  int rc = 0;
  if (!current_sms(&rc)) return rc;
  return launch_status(fitq::launch_lora_merge(w, w_dtype, n_out, k_in, lora_a, lora_b, rank, scale,
                                               static_cast<cudaStream_t>(stream)),
                       "lora_merge");
}

size_t fitq_nf4_down_dswiglu_workspace(int64_t m, int64_t n_out, int64_t k_in) {
  (void)m;
  Carve c{nullptr, 0};
  c.take(bf16_bytes(n_out * k_in));
  return c.used;
}

int fitq_nf4_down_dswiglu(const fitq_nf4_weight* w_down, const void* dy, int64_t m, const void* gate,
                          const void* up, void* d_gate, void* d_up, void* workspace,
                          size_t workspace_bytes, fitq_stream_t stream) {
  fitq::Nf4Args a;
  int rc = check_weight(w_down, &a);
  if (rc) return rc;
  if (!dy || !gate || !up || !d_gate || !d_up)
    return fail(FITQ_ERR_ARG, "down_dswiglu: dy, gate, up, d_gate and d_up are required");
  if (m <= 0 || m >= (1ll << 31)) return fail(FITQ_ERR_SHAPE, "down_dswiglu: bad M=%lld", (long long)m);
  const int64_t N = a.n_out, K = a.k_in;  // dX [M, K] = dy [M, N] . W [N, K]
  if (N % 64 != 0 || K % 16 != 0)
    return fail(FITQ_ERR_SHAPE, "down_dswiglu: need N %% 64 == 0 and K %% 16 == 0 (N=%lld K=%lld)",
                (long long)N, (long long)K);
  if (!al16(dy) || !al16(gate) || !al16(up) || !al16(d_gate) || !al16(d_up))
    return fail(FITQ_ERR_ALIGN, "down_dswiglu: 16-byte alignment");
  const size_t need = fitq_nf4_down_dswiglu_workspace(m, N, K);
  if (!workspace || workspace_bytes < need)
    return fail(FITQ_ERR_WORKSPACE, "down_dswiglu: workspace %zu < %zu bytes", workspace_bytes, need);
  int sms = current_sms(&rc);
  if (!sms) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if ((rc = fitq::launch_nf4_dequant(a, workspace, FITQ_DTYPE_BF16, 1, st, sms)))
    return launch_status(rc, "nf4_dequant (transposed)");
  fitq::GemmArgs g{};
  g.a = dy; g.lda = N;
  g.b = workspace; g.ldb = N;
  g.c = d_gate; g.ldc = K;
  g.m = m; g.n = K; g.k = N;
  g.epi = fitq::GEMM_EPI_DSWIGLU;
  g.src0 = gate; g.src1 = up; g.aux0 = d_up;
  g.status = status_ptr();
  return launch_status(fitq::launch_gemm(g, st, sms), "tcgen05 gemm (down dX + SwiGLU backward)");
}

int fitq_gemm_bf16_tn(const void* a, const void* b, void* c, const void* c_add, int64_t m,
                      int64_t n, int64_t k, fitq_stream_t stream) {
  if (!a || !b || !c) return fail(FITQ_ERR_ARG, "gemm: NULL operand");
  if (m <= 0 || n <= 0 || k <= 0 || k % 64 != 0 || n % 16 != 0 || m >= (1ll << 31) ||
      n >= (1ll << 31) || k >= (1ll << 31))
    return fail(FITQ_ERR_SHAPE, "gemm: need K %% 64 == 0 and N %% 16 == 0 (M=%lld N=%lld K=%lld)",
                (long long)m, (long long)n, (long long)k);
  if (!al16(a) || !al16(b) || !al16(c) || (c_add && !al16(c_add)))
    return fail(FITQ_ERR_ALIGN, "gemm: operands must be 16-byte aligned");
  int rc;
  int sms = current_sms(&rc);
  if (!sms) return rc;
  fitq::GemmArgs g{};
  g.a = a; g.lda = k;
  g.b = b; g.ldb = k;
  g.c = c; g.ldc = n;
  g.c_add = c_add; g.ldc_add = n;
  g.m = m; g.n = n; g.k = k;
  g.lora_k = 0;
  g.status = status_ptr();
  return launch_status(fitq::launch_gemm(g, static_cast<cudaStream_t>(stream), sms),
                       "tcgen05 gemm");
}

int fitq_adamw_step(float* param, const float* grad, float* exp_avg, float* exp_avg_sq,
                    int64_t n, float lr, float beta1, float beta2, float eps,
                    float weight_decay, int step, const float* clip, fitq_stream_t stream) {
  if (!param || !grad || !exp_avg || !exp_avg_sq) return fail(FITQ_ERR_ARG, "adamw: NULL buffer");
  if (n < 0 || step < 1) return fail(FITQ_ERR_ARG, "adamw: need n >= 0 and step >= 1");
  int rc;
  if (!current_sms(&rc)) return rc;
  if (n == 0) return FITQ_OK;
  return launch_status(fitq::launch_adamw(param, grad, exp_avg, exp_avg_sq, n, lr, beta1, beta2,
                                          eps, weight_decay, step, clip,
                                          static_cast<cudaStream_t>(stream)),
                       "adamw");
}

size_t fitq_grad_norm_workspace(int64_t n) { return fitq::grad_norm_workspace(n); }

int fitq_grad_clip_coef(const float* grads, int64_t n, float max_norm, float* norm_out,
                        void* workspace, size_t workspace_bytes, fitq_stream_t stream) {
  if (!grads || !norm_out) return fail(FITQ_ERR_ARG, "grad_clip: NULL buffer");
  if (n < 0) return fail(FITQ_ERR_ARG, "grad_clip: n < 0");
  const size_t need = fitq::grad_norm_workspace(n);
  if (!workspace || workspace_bytes < need)
    return fail(FITQ_ERR_WORKSPACE, "grad_clip: workspace %zu < %zu bytes", workspace_bytes, need);
  int rc;
  if (!current_sms(&rc)) return rc;
  return launch_status(fitq::launch_grad_clip(grads, n, max_norm, norm_out, workspace,
                                              static_cast<cudaStream_t>(stream)),
                       "grad_clip");
}

}  // extern "C"

// ---------------------------------------------------------------- launch timing
// One process-wide table of CUDA event pairs (events are host handles; no
// device memory is allocated).  Recording is off unless fitq_timing_enable()
// was called with a positive capacity.
namespace {
struct TimingTable {
  std::vector<cudaEvent_t> start, stop;
  std::vector<double> flops;
  int used = 0;
  int capacity = 0;
};
TimingTable g_timing;
std::mutex g_timing_mu;
}  // namespace

namespace fitq {
int timing_begin(cudaStream_t st, double flops) {
  std::lock_guard<std::mutex> lk(g_timing_mu);
  if (g_timing.used >= g_timing.capacity) return -1;
  const int slot = g_timing.used++;
  g_timing.flops[slot] = flops;
  cudaEventRecord(g_timing.start[slot], st);
  return slot;
}
void timing_end(int slot, cudaStream_t st) {
  if (slot < 0) return;
  cudaEventRecord(g_timing.stop[slot], st);
}
}  // namespace fitq

extern "C" {

int fitq_timing_enable(int capacity) {
  std::lock_guard<std::mutex> lk(g_timing_mu);
  if (capacity < 0) return fail(FITQ_ERR_ARG, "timing: negative capacity");
  if (static_cast<size_t>(capacity) > g_timing.start.size()) {
    int code;
    if (!current_sms(&code)) return code;
    while (g_timing.start.size() < static_cast<size_t>(capacity)) {
      cudaEvent_t a, b;
      if (cudaEventCreate(&a) != cudaSuccess || cudaEventCreate(&b) != cudaSuccess)
        return fail(FITQ_ERR_CUDA, "timing: cudaEventCreate failed");
      g_timing.start.push_back(a);
      g_timing.stop.push_back(b);
      g_timing.flops.push_back(0.0);
    }
  }
  g_timing.capacity = capacity;
  g_timing.used = 0;
  return FITQ_OK;
}

int fitq_timing_read(float* ms, double* flops, int max) {
  std::lock_guard<std::mutex> lk(g_timing_mu);
  const int n = g_timing.used < max ? g_timing.used : max;
  for (int i = 0; i < n; ++i) {
    if (cudaEventSynchronize(g_timing.stop[i]) != cudaSuccess)
      return -fail(FITQ_ERR_CUDA, "timing: event sync failed");
    float t = 0.f;
    cudaEventElapsedTime(&t, g_timing.start[i], g_timing.stop[i]);
    if (ms) ms[i] = t;
    if (flops) flops[i] = g_timing.flops[i];
  }
  return n;
}

}  // extern "C"

namespace {
std::atomic<long long> g_launches{0};
}
namespace fitq {
void note_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

bool set_smem_limit(const void* fn, int bytes) {
  static std::mutex mu;
  static std::vector<std::pair<int, const void*>> done;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return false;
  std::lock_guard<std::mutex> lk(mu);
  for (const auto& d : done)
    if (d.first == dev && d.second == fn) return true;
  if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) != cudaSuccess)
    return false;
  done.emplace_back(dev, fn);
  return true;
}
}  // namespace fitq
extern "C" long long fitq_launch_count(void) { return g_launches.load(); }

namespace fitq {
// Lets entry points defined in other files report through fitq_last_error().
void set_last_error(const char* msg) { g_last_error = msg; }
void note_launch_detail(const char* msg) { g_launch_detail = msg; }
int launch_result() {
  const cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) return FITQ_OK;
  g_launch_error = e;
  return FITQ_ERR_CUDA;
}
}  // namespace fitq

// ---------------------------------------------------------------- layer kernels
extern "C" {

int fitq_rmsnorm_fwd(const void* x, const void* weight, void* y, int64_t rows, int64_t cols,
                     float eps, fitq_stream_t stream) {
  if (!x || !weight || !y) return fail(FITQ_ERR_ARG, "rmsnorm: NULL tensor");
  if (rows <= 0 || cols <= 0 || cols % 8 != 0 || rows >= (1ll << 31))
    return fail(FITQ_ERR_SHAPE, "rmsnorm: need cols %% 8 == 0 (rows=%lld cols=%lld)",
                (long long)rows, (long long)cols);
  if (!al16(x) || !al16(weight) || !al16(y)) return fail(FITQ_ERR_ALIGN, "rmsnorm: 16-byte alignment");
  int rc;
  if (!current_sms(&rc)) return rc;
  return launch_status(fitq::launch_rmsnorm_fwd(x, weight, y, rows, cols, eps,
                                                static_cast<cudaStream_t>(stream)), "rmsnorm_fwd");
}

int fitq_rmsnorm_bwd(const void* dy, const void* x, const void* weight, void* dx, int64_t rows,
                     int64_t cols, float eps, fitq_stream_t stream) {
  if (!dy || !x || !weight || !dx) return fail(FITQ_ERR_ARG, "rmsnorm_bwd: NULL tensor");
  if (rows <= 0 || cols <= 0 || cols % 8 != 0 || rows >= (1ll << 31))
    return fail(FITQ_ERR_SHAPE, "rmsnorm_bwd: need cols %% 8 == 0");
  if (!al16(dy) || !al16(x) || !al16(weight) || !al16(dx))
    return fail(FITQ_ERR_ALIGN, "rmsnorm_bwd: 16-byte alignment");
  int rc;
  if (!current_sms(&rc)) return rc;
  return launch_status(fitq::launch_rmsnorm_bwd(dy, x, weight, dx, rows, cols, eps,
                                                static_cast<cudaStream_t>(stream)), "rmsnorm_bwd");
}

int fitq_rope(const void* t, void* out, const float* cos_half, const float* sin_half, int64_t rows,
              int heads, int head_dim, int64_t seq, int backward, fitq_stream_t stream) {
  if (!t || !out || !cos_half || !sin_half) return fail(FITQ_ERR_ARG, "rope: NULL tensor");
  if (rows <= 0 || heads <= 0 || head_dim <= 0 || head_dim % 16 != 0 || seq <= 0)
    return fail(FITQ_ERR_SHAPE, "rope: need head_dim %% 16 == 0");
  if (!al16(t) || !al16(out) || !al16(cos_half) || !al16(sin_half))
    return fail(FITQ_ERR_ALIGN, "rope: 16-byte alignment");
  int rc;
  const int sms = current_sms(&rc);
  if (!sms) return rc;
  return launch_status(fitq::launch_rope(t, out, cos_half, sin_half, rows, heads, head_dim, seq,
                                         backward, static_cast<cudaStream_t>(stream), sms), "rope");
}

size_t fitq_cross_entropy_workspace(int64_t rows) {
  return rows > 0 ? fitq::cross_entropy_workspace(rows) : 0;
}

int fitq_cross_entropy(void* logits, const int64_t* labels, int64_t rows, int64_t vocab,
                       int64_t ignore_index, float loss_scale, float* loss_out, void* workspace,
                       size_t workspace_bytes, fitq_stream_t stream) {
  if (!logits || !labels || !loss_out || !workspace)
    return fail(FITQ_ERR_ARG, "cross_entropy: NULL tensor or workspace");
  if (rows <= 0 || rows >= (1ll << 31) || vocab <= 0 || vocab % 8 != 0)
    return fail(FITQ_ERR_SHAPE, "cross_entropy: need rows > 0 and vocab %% 8 == 0 (rows=%lld V=%lld)",
                (long long)rows, (long long)vocab);
  if (!al16(logits) || (reinterpret_cast<uintptr_t>(labels) & 7) != 0 || !al16(workspace))
    return fail(FITQ_ERR_ALIGN, "cross_entropy: alignment");
  if (workspace_bytes < fitq::cross_entropy_workspace(rows))
    return fail(FITQ_ERR_WORKSPACE, "cross_entropy: workspace %zu < %zu bytes", workspace_bytes,
                fitq::cross_entropy_workspace(rows));
  int rc;
  if (!current_sms(&rc)) return rc;
  return launch_status(fitq::launch_cross_entropy(logits, labels, rows, vocab, ignore_index, loss_scale,
                                                  loss_out, workspace, static_cast<cudaStream_t>(stream)),
                       "cross_entropy");
}

size_t fitq_verify_attention_workspace(int64_t batch, int heads, int kv_heads, int t_new,
                                       int prefix) {
  (void)heads;
  int rc;
  const int sms = current_sms(&rc);
  if (!sms || batch <= 0 || kv_heads <= 0 || t_new <= 0 || prefix < 0) return 0;
  return fitq::verify_attention_workspace(batch, kv_heads, prefix + t_new, sms);
}

int fitq_verify_attention(const void* q, const void* k_cache, const void* v_cache, void* out,
                          int64_t batch, int heads, int kv_heads, int t_new, int prefix,
                          int capacity, int head_dim, void* workspace, size_t workspace_bytes,
                          fitq_stream_t stream) {
  if (!q || !k_cache || !v_cache || !out || !workspace)
    return fail(FITQ_ERR_ARG, "verify_attention: NULL tensor or workspace");
  if (batch <= 0 || batch > 65535 || heads <= 0 || kv_heads <= 0 || heads % kv_heads != 0 ||
      kv_heads > 65535 || t_new <= 0 || prefix < 0 || prefix + t_new > capacity)
    return fail(FITQ_ERR_SHAPE, "verify_attention: bad shape (B=%lld H=%d KVH=%d T=%d prefix=%d cap=%d)",
                (long long)batch, heads, kv_heads, t_new, prefix, capacity);
  if (head_dim != 128 || (heads / kv_heads) * t_new > 32)
    return fail(FITQ_ERR_UNSUPPORTED,
                "verify_attention: needs head_dim 128 and (H / KVH) * T <= 32 (D=%d G*T=%d)", head_dim,
                (heads / kv_heads) * t_new);
  if (!al16(q) || !al16(k_cache) || !al16(v_cache) || !al16(out) || !al16(workspace))
    return fail(FITQ_ERR_ALIGN, "verify_attention: 16-byte alignment");
  int rc;
  const int sms = current_sms(&rc);
  if (!sms) return rc;
  const size_t need = fitq::verify_attention_workspace(batch, kv_heads, prefix + t_new, sms);
  if (workspace_bytes < need)
    return fail(FITQ_ERR_WORKSPACE, "verify_attention: workspace %zu < %zu bytes", workspace_bytes, need);
  return launch_status(fitq::launch_verify_attention(q, k_cache, v_cache, out, batch, heads, kv_heads,
                                                     t_new, prefix, capacity, workspace,
                                                     static_cast<cudaStream_t>(stream), sms),
                       "verify_attention");
}

// Shape checks shared by the training attention forward and backward.
static int attention_shape(const char* what, int64_t batch, int64_t seq, int heads, int kv_heads,
                           int head_dim) {
  if (batch <= 0 || batch > 65535 || seq <= 0 || seq % 64 != 0 || seq > (1ll << 30) || heads <= 0 ||
      heads > 65535 || kv_heads <= 0 || heads % kv_heads != 0)
    return fail(FITQ_ERR_SHAPE, "%s: bad shape (B=%lld S=%lld H=%d KVH=%d; S %% 64 == 0, H %% KVH == 0)",
                what, (long long)batch, (long long)seq, heads, kv_heads);
  if (head_dim != 128) return fail(FITQ_ERR_UNSUPPORTED, "%s: needs head_dim 128 (got %d)", what, head_dim);
  return FITQ_OK;
}

int fitq_attention_fwd(const void* q, const void* k, const void* v, void* o, float* lse,
                       int64_t batch, int64_t seq, int heads, int kv_heads, int head_dim,
                       fitq_stream_t stream) {
  if (!q || !k || !v || !o || !lse) return fail(FITQ_ERR_ARG, "attention_fwd: NULL tensor");
  int rc = attention_shape("attention_fwd", batch, seq, heads, kv_heads, head_dim);
  if (rc) return rc;
  if (!al16(q) || !al16(k) || !al16(v) || !al16(o) || !al16(lse))
    return fail(FITQ_ERR_ALIGN, "attention_fwd: 16-byte alignment");
  if (!current_sms(&rc)) return rc;
  return launch_status(fitq::launch_train_attn_fwd(q, k, v, o, lse, batch, seq, heads, kv_heads,
                                                   static_cast<cudaStream_t>(stream)),
                       "attention_fwd");
}

size_t fitq_attention_bwd_workspace(int64_t batch, int64_t seq, int heads) {
  if (batch <= 0 || seq <= 0 || heads <= 0) return 0;
  return static_cast<size_t>(batch) * static_cast<size_t>(seq) * static_cast<size_t>(heads) * sizeof(float);
}

int fitq_attention_bwd(const void* q, const void* k, const void* v, const void* o, const void* d_o,
                       const float* lse, void* dq, void* dk, void* dv, int64_t batch, int64_t seq,
                       int heads, int kv_heads, int head_dim, void* workspace, size_t workspace_bytes,
                       fitq_stream_t stream) {
  if (!q || !k || !v || !o || !d_o || !lse || !dq || !dk || !dv || !workspace)
    return fail(FITQ_ERR_ARG, "attention_bwd: NULL tensor or workspace");
  int rc = attention_shape("attention_bwd", batch, seq, heads, kv_heads, head_dim);
  if (rc) return rc;
  if (!al16(q) || !al16(k) || !al16(v) || !al16(o) || !al16(d_o) || !al16(lse) || !al16(dq) ||
      !al16(dk) || !al16(dv) || !al16(workspace))
    return fail(FITQ_ERR_ALIGN, "attention_bwd: 16-byte alignment");
  const size_t need = fitq_attention_bwd_workspace(batch, seq, heads);
  if (workspace_bytes < need)
    return fail(FITQ_ERR_WORKSPACE, "attention_bwd: workspace %zu < %zu bytes", workspace_bytes, need);
  if (!current_sms(&rc)) return rc;
  return launch_status(fitq::launch_train_attn_bwd(q, k, v, o, d_o, lse, dq, dk, dv,
                                                   static_cast<float*>(workspace), batch, seq, heads,
                                                   kv_heads, static_cast<cudaStream_t>(stream)),
                       "attention_bwd");
}

int fitq_rope_append(const void* q, const void* k, const void* v, void* q_out, void* k_cache,
                     void* v_cache, const float* cos_half, const float* sin_half, int64_t batch,
                     int t_new, int heads, int kv_heads, int head_dim, int prefix, int capacity,
                     fitq_stream_t stream) {
  if (!q || !k || !v || !q_out || !k_cache || !v_cache || !cos_half || !sin_half)
    return fail(FITQ_ERR_ARG, "rope_append: NULL tensor");
  if (batch <= 0 || t_new <= 0 || heads <= 0 || kv_heads <= 0 || head_dim <= 0 || head_dim % 16 != 0 ||
      prefix < 0 || prefix + t_new > capacity)
    return fail(FITQ_ERR_SHAPE, "rope_append: bad shape (head_dim %% 16 == 0, prefix + T <= capacity)");
  if (!al16(q) || !al16(k) || !al16(v) || !al16(q_out) || !al16(k_cache) || !al16(v_cache) ||
      !al16(cos_half) || !al16(sin_half))
    return fail(FITQ_ERR_ALIGN, "rope_append: 16-byte alignment");
  int rc;
  const int sms = current_sms(&rc);
  if (!sms) return rc;
  return launch_status(fitq::launch_rope_append(q, k, v, q_out, k_cache, v_cache, cos_half, sin_half,
                                                batch, t_new, heads, kv_heads, head_dim, prefix,
                                                capacity, static_cast<cudaStream_t>(stream), sms),
                       "rope_append");
}

int fitq_swiglu_fwd(const void* gate, const void* up, void* act, int64_t n, fitq_stream_t stream) {
  if (!gate || !up || !act) return fail(FITQ_ERR_ARG, "swiglu: NULL tensor");
  if (n <= 0 || n % 8 != 0) return fail(FITQ_ERR_SHAPE, "swiglu: need n %% 8 == 0");
  if (!al16(gate) || !al16(up) || !al16(act)) return fail(FITQ_ERR_ALIGN, "swiglu: 16-byte alignment");
  int rc;
  const int sms = current_sms(&rc);
  if (!sms) return rc;
  return launch_status(fitq::launch_swiglu_fwd(gate, up, act, n, static_cast<cudaStream_t>(stream), sms),
                       "swiglu_fwd");
}

int fitq_swiglu_bwd(const void* d_act, const void* gate, const void* up, void* d_gate, void* d_up,
                    int64_t n, fitq_stream_t stream) {
  if (!d_act || !gate || !up || !d_gate || !d_up) return fail(FITQ_ERR_ARG, "swiglu_bwd: NULL tensor");
  if (n <= 0 || n % 8 != 0) return fail(FITQ_ERR_SHAPE, "swiglu_bwd: need n %% 8 == 0");
  if (!al16(d_act) || !al16(gate) || !al16(up) || !al16(d_gate) || !al16(d_up))
    return fail(FITQ_ERR_ALIGN, "swiglu_bwd: 16-byte alignment");
  int rc;
  const int sms = current_sms(&rc);
  if (!sms) return rc;
  return launch_status(fitq::launch_swiglu_bwd(d_act, gate, up, d_gate, d_up, n,
                                               static_cast<cudaStream_t>(stream), sms),
                       "swiglu_bwd");
}

}  // extern "C"
