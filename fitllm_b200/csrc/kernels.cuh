// Internal launcher declarations shared by the .cu files of libfitq.
#pragma once
#include <cstdint>
#include <cstdlib>
#include <cuda.h>
#include <cuda_runtime.h>

#include "../../include/fitq.h"

namespace fitq {

constexpr int64_t kOffsetChunk = 4096;  // absmax mean: double sum per chunk, then chunks in order

// Device-side copy of fitq_nf4_weight.
struct Nf4Args {
  const uint8_t* packed;
  const uint8_t* absmax_code;
  const float* nested_absmax;
  const float* nested_quant_map;
  const float* absmax_f32;
  const float* quant_map;
  float offset;
  int64_t n_out;
  int64_t k_in;
};

int launch_nf4_dequant(const Nf4Args& w, void* out, int out_dtype, int transpose, cudaStream_t st,
                       int num_sms);
int launch_nf4_quantize(const float* wt, int64_t n, const float* qmap, const float* nqmap,
                        uint8_t* packed, uint8_t* codes, float* nested_absmax, float* offset_out,
                        float* absmax_ws, double* partial_ws, cudaStream_t st, int num_sms);

// tcgen05 GEMM: C[M,N] = A[M,K].B[N,K]^T (+ Pa[M,r].Pb[N,r]^T) (+ C_add).
// A/B/Pa/Pb bf16 row-major; Pa/Pb have a row pitch of 64 elements, columns
// r..63 ignored.  lora_k in {0,16,32,48,64}.
struct GemmArgs {
  const void* a; int64_t lda;
  const void* b; int64_t ldb;
  const void* pa;  // may be null when lora_k == 0
  const void* pb;
  void* c; int64_t ldc;
  const void* c_add; int64_t ldc_add;
  const void* bias;  // bf16 [N] or null
  int64_t m, n, k;
  int lora_k;
  int* status;  // device status word (bounded-wait timeouts)
  // Epilogue modes of the pair kernel (launch_gemm_bf16_tn_2cta):
  //   GEMM_EPI_SWIGLU: gate and up in one launch -- b = W_gate, b2 = W_up
  //     (bf16 [n, k] each, pitch ldb); c[m, n] = silu(g) * u of the
  //     bf16-rounded products g = a.W_gate^T, u = a.W_up^T; g, u also stored
  //     into aux0 / aux1 (pitch ldc) when non-null.  No LoRA, bias or c_add.
  //   GEMM_EPI_DSWIGLU: with d = bf16(a.b^T), g = src0, u = src1 (bf16
  //     [m, n], pitch ldc): c = d(silu(g) * u)/dg, aux0 = .../du.
  int epi;
  const void* b2;
  const void* src0;
  const void* src1;
  void* aux0;
  void* aux1;
};
constexpr int GEMM_EPI_PLAIN = 0, GEMM_EPI_SWIGLU = 1, GEMM_EPI_DSWIGLU = 2;
int launch_gemm_bf16_tn(const GemmArgs& g, cudaStream_t st, int num_sms);
// Same contract on CTA pairs (cta_group::2, 256x256 tiles), gemm_sm100_2cta.cu.
int launch_gemm_bf16_tn_2cta(const GemmArgs& g, cudaStream_t st, int num_sms);
// Picks the pair kernel when there are enough 256x256 tiles to fill the GPU
// (FITQ_GEMM_VARIANT=1cta|2cta in the environment forces one).
int launch_gemm(const GemmArgs& g, cudaStream_t st, int num_sms);

// NF4 dequant fused into the tcgen05 GEMM (gemm_nf4.cu): the weight operand
// is decoded bit-exactly from the packed codes into shared memory.
//   trans = 0: C[m, N_w] = A[m, K_w] . W_deq^T   (A = x, forward)
//   trans = 1: C[m, K_w] = A[m, N_w] . W_deq     (A = dy, input gradient)
// plus the LoRA K-block pa[m, r] . pb[cols, r]^T (bf16, pitch 64) and the
// bias / residual epilogue of GemmArgs.  Needs the GEMM's output columns % 128
// == 0 and its reduction % 64 == 0 (gemm_nf4_shape_ok).
struct Nf4GemmArgs {
  Nf4Args w;
  int trans;
  const void* a; int64_t lda;
  const void* pa;
  const void* pb;
  void* c; int64_t ldc;
  const void* c_add; int64_t ldc_add;
  const void* bias;
  int64_t m;
  int lora_k;
  int* status;
};
inline bool gemm_nf4_shape_ok(int64_t n_out, int64_t k_in, int trans) {
  const int64_t cols = trans ? k_in : n_out, red = trans ? n_out : k_in;
  return cols % 128 == 0 && red % 64 == 0 && k_in % 64 == 0;
}
bool gemm_nf4_supported(const Nf4Args& w, int trans);
// Picks the CTA-pair kernel (256 x 256 tiles, gemm_nf4_2cta.cu) when the
// output columns are a multiple of 256, else the one-CTA kernel (256 x 128
// tiles); FITQ_NF4_GEMM=1cta in the environment forces the one-CTA kernel.
int launch_gemm_nf4(const Nf4GemmArgs& g, cudaStream_t st, int num_sms);
bool gemm_nf4_2cta_supported(const Nf4Args& w, int trans);
int launch_gemm_nf4_2cta(const Nf4GemmArgs& g, cudaStream_t st, int num_sms);

// LoRA building blocks (lora.cu).
// out[M, r] = in[M, D] . wt[r, D]^T  (bf16 in, fp32 accumulate); written as
// bf16 into out_pad (row pitch 64; columns r..63 are left untouched and never
// read, since r % 16 == 0) and, when non-null, into out_dense [M, r].
// Launch with programmatic stream serialisation (see pdl_wait in common.cuh)
// unless FITQ_PDL=0 is set in the environment.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                       cudaStream_t st, Args... args) {
  static const bool off = [] {
    const char* e = getenv("FITQ_PDL");
    return e != nullptr && e[0] == '0';
  }();
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = off ? 0 : 1;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

// Partials of T = x.A^T for M <= 64 rows in one launch (lora.cu): bf16 x
// [M, K], fp32 A [r, K] (rounded to bf16 like autocast does), fp32
// accumulate; part_ws [K/64][M][r] fp32 (lora_t_workspace bytes), summed in
// group order by the decode finishing kernel.  K % 64 == 0, r % 4 == 0.
// Must be launched right behind launch_nf4_gemv_dec (it reads x without
// waiting).
size_t lora_t_workspace(int64_t M, int64_t K, int r);
int lora_t_groups(int64_t K);
int launch_lora_t(const void* x, int64_t M, int64_t K, const float* a, int r, float* part_ws,
                  cudaStream_t st);
// The same for 1-3 (A, rank, partials) jobs on one x in one launch.
int launch_lora_t_multi(const void* x, int64_t M, int64_t K, const float* const* a, const int* r,
                        float* const* part_ws, int jobs, cudaStream_t st);

int launch_lora_rowproj(const void* in, int64_t ld_in, int64_t M, int64_t D, const void* wt_bf16,
                        int r, void* out_pad, void* out_dense, cudaStream_t st, int num_sms);
// The same projection for few rows (M <= 64): D split over CTAs, fp32
// partials in partial_ws (lora_rowproj_small_workspace bytes), reduced in
// slice order into out_pad (pitch 64) and out_dense.
size_t lora_rowproj_small_workspace(int64_t M, int64_t D, int r);
int launch_lora_rowproj_small(const void* in, int64_t ld_in, int64_t M, int64_t D,
                              const void* wt_bf16, int r, float* partial_ws, void* out_pad,
                              void* out_dense, cudaStream_t st);
// Reduction over rows:  res[r, D] = scale . p[M, r]^T . in[M, D]
// (p bf16 with row pitch ld_p, a multiple of 8).  layout 0 writes res[r][D],
// layout 1 res[D][r].  accumulate != 0 adds into res.  partial_ws: fp32
// [chunks, r, D] scratch of lora_colproj_workspace() bytes.
size_t lora_colproj_workspace(int64_t M, int64_t D, int r, int num_sms);
int launch_lora_colproj(const void* p, int64_t ld_p, const void* in, int64_t ld_in, int64_t M, int64_t D,
                        int r, float scale, float* res, int layout, int accumulate,
                        float* partial_ws, cudaStream_t st, int num_sms);
// fp32 [rows, r] (row-major) -> bf16 scaled, pitch 64, zero padded: out[i][j] = bf16(s*in[i][j]).
int launch_pad_lora_weight(const float* in, int64_t rows, int r, float scale, int transpose_in,
                           void* out_pad, cudaStream_t st);
// fp32 -> bf16 copy of a [r, D] matrix.
int launch_f32_to_bf16(const float* in, int64_t n, void* out, cudaStream_t st);
// fp32 [rows, cols] -> bf16 [cols, rows] (transposed).
int launch_f32_to_bf16_t(const float* in, int64_t rows, int cols, void* out, cudaStream_t st);

// NF4 decode GEMV for M <= 8 (gemv.cu): y = sum + scale * T.B^T + bias +
// y_add (bf16) in the kernel when K is one slice; otherwise fp32 split-K
// partials and a finishing launch right behind it (programmatic dependent
// launch).
struct GemvEpilogue {
  void* y;               // bf16 [M, N]
  const void* y_add;     // bf16 [M, N] or null
  const void* bias;      // bf16 [N] or null
  const float* lora_b;   // fp32 [N, rank] or null
  const float* t_part;   // fp32 [t_groups, M, rank] partials of T = x.A^T, or null
  int t_groups;
  void* t_dense;         // bf16 [M, rank]: receives T when non-null
  int rank;
  float scale;
  float* partial;        // fp32 [slices, M, N] when the finishing kernel runs
};
// Up to three weights with one K streamed by one decode launch (the q/k/v or
// gate/up projections of a layer on the same x): tiles (16 rows)
// [tile0[j], tile0[j + 1]) are weight j's; tile0[3] = all tiles.  Weight j
// writes fp32 partials [slices, M, N_j] to partial[j] (null: the single-weight
// launch writes y through its epilogue).  status: where a grouped launch whose
// weights carry different code tables reports FITQ_ERR_UNSUPPORTED.
struct DecJobs {
  Nf4Args w[3];
  float* partial[3];
  int tile0[4];
  int groups;
  int* status;
};
// True when the decode kernel takes (m, N, K); *slices = its K slices.
bool gemv_dec_plan(int64_t m, int64_t n_out, int64_t k_in, int num_sms, int* slices);
// Whether the decode GEMV writes fp32 partials (several K slices, or a LoRA
// term: T is computed while the weights stream) and needs the finishing
// launch; the order is launch_nf4_gemv_dec, launch_lora_t (rank > 0), then
// launch_nf4_gemv_dec_finish.
bool gemv_dec_needs_partial(int slices, int rank);
int launch_nf4_gemv_dec(const Nf4Args& w, const void* x, int64_t m, const GemvEpilogue& out,
                        cudaStream_t st, int num_sms);
// The decode kernel over 1-3 weights sharing K and x (partials only; the plan
// of the summed N: gemv_dec_plan(m, sum N, K, ...)).
int launch_nf4_gemv_dec_grouped(const Nf4Args* w, int groups, const void* x, int64_t m,
                                float* const* partial, int* status, cudaStream_t st, int num_sms);
int launch_nf4_gemv_dec_finish(int64_t m, int64_t n_out, int slices, const GemvEpilogue& out,
                               cudaStream_t st, int num_sms);
// The finishing pass of a grouped launch (up to three epilogues, one grid);
// with swiglu_act (two projections of equal N, rank 0) only
// act = SwiGLU(first, second) is stored, bf16 [M, N].
int launch_nf4_gemv_group_finish(int64_t m, const int64_t* n_out, int jobs, int slices,
                                 const GemvEpilogue* eps, void* swiglu_act, cudaStream_t st);

// 2-D tiled tensor map [outer rows][inner elements], row pitch row_bytes; elements
// outside the tensor read as zero (gemm_sm100.cu).
bool encode_tmap_2d(CUtensorMap* m, CUtensorMapDataType dtype, const void* base, uint64_t inner,
                    uint64_t outer, uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer,
                    CUtensorMapSwizzle swizzle, CUtensorMapL2promotion l2);

// NF4 skinny GEMM on tcgen05 with the decoded weights in tensor memory
// (gemv_tc.cu), 8 < M <= 64 (FITQ_GEMV_TC=1: also M <= 8, =0: never);
// N % 128 == 0, K % 256 == 0, packed weights and x 16-byte aligned.  Writes
// fp32 split-K partials [slices, M, N] for launch_nf4_gemv_dec_finish.
bool gemv_tc_plan(int64_t m, int64_t n_out, int64_t k_in, int num_sms, int* slices);
int launch_nf4_gemv_tc(const Nf4Args& w, const void* x, int64_t m, float* partial, int* status,
                       cudaStream_t st, int num_sms);
// One launch over up to three weights sharing K, x and the scale format (q/k/v,
// gate/up): partial[g] = [slices, M, N_g] with the slices gemv_tc_plan gives for
// N = the sum of the N_g.
int launch_nf4_gemv_tc_grouped(const Nf4Args* w, int groups, const void* x, int64_t m,
                               float* const* partial, int* status, cudaStream_t st, int num_sms);

// Cross-entropy of [T, V] bf16 logits, mean over labels != ignore_index; the
// logits are overwritten with d(loss_scale * loss)/dlogits (ce.cu).
size_t cross_entropy_workspace(int64_t rows);
int launch_cross_entropy(void* logits, const int64_t* labels, int64_t T, int64_t V,
                         int64_t ignore_index, float loss_scale, float* loss_out, void* workspace,
                         cudaStream_t st);

// Speculative-verify attention over a KV cache (attn.cu): q, out [B, T, H, 128],
// caches [B, KVH, cap, 128] bf16, (H / KVH) * T <= 32, prefix + T <= cap.
// Causal GQA attention of the training layer (train_attn.cu); shapes checked
// by the caller: head_dim 128, seq % 64 == 0, heads % kv_heads == 0.
int launch_train_attn_fwd(const void* q, const void* k, const void* v, void* out, float* lse,
                          int64_t batch, int64_t seq, int heads, int kv_heads, cudaStream_t st);
int launch_train_attn_bwd(const void* q, const void* k, const void* v, const void* o,
                          const void* d_o, const float* lse, void* dq, void* dk, void* dv,
                          float* delta, int64_t batch, int64_t seq, int heads, int kv_heads,
                          cudaStream_t st);
size_t verify_attention_workspace(int64_t batch, int kv_heads, int len, int num_sms);
int launch_verify_attention(const void* q, const void* k_cache, const void* v_cache, void* out,
                            int64_t batch, int heads, int kv_heads, int t_new, int prefix, int cap,
                            void* workspace, cudaStream_t st, int num_sms);

// NF4 GEMV / skinny GEMM for M <= 64 (gemv.cu): split-K partial products
// [splits, M, N] fp32, then a finishing pass adding LoRA / y_add -> bf16.
size_t gemv_partial_bytes(int64_t m, int64_t n_out, int64_t k_in, int num_sms, int* splits_out);
int launch_nf4_gemv_core(const Nf4Args& w, const void* x, int64_t m, float* partial,
                         cudaStream_t st, int num_sms, int* splits_out);
int launch_gemv_finish(const float* partial, int splits, int64_t m, int64_t n, const void* t_pad,
                       const float* lora_b, int rank, float scale, const void* bias,
                       const void* y_add, void* y, cudaStream_t st, int num_sms);

// Launch timing of the tcgen05 GEMM (abi.cu): when enabled, CUDA events are
// recorded on the launching stream around each launch.  timing_begin returns
// a slot (or -1 when disabled / full); timing_end records the stop event.
int timing_begin(cudaStream_t st, double flops);
// Counts kernel launches made by the library (read by fitq_launch_count).
void note_launch();
// Raise a kernel's dynamic shared-memory limit to `bytes` on the current
// device, once per (device, kernel): kernel attributes belong to a device's
// context, so a process that drives several GPUs sets them on each.  False
// when CUDA refuses.
bool set_smem_limit(const void* fn, int bytes);
template <typename F>
bool set_smem_limit(F* fn, int bytes) {
  return set_smem_limit(reinterpret_cast<const void*>(fn), bytes);
}
// W[n,k] (bf16 / fp16, in place) += scale * (B[n,:] . A[:,k]); see merge.cu.
int launch_lora_merge(void* w, int out_dtype, int64_t n, int64_t k, const float* a, const float* b,
                      int rank, float scale, cudaStream_t st);

// One thread waits with mbar_wait_for on an mbarrier nothing completes; after
// limit_ns it records FITQ_ERR_TIMEOUT in *status and returns (selftest.cu).
int launch_selftest_wait(uint64_t limit_ns, unsigned long long* elapsed_ns, int* status,
                         cudaStream_t st);
// Sets the text returned by fitq_last_error() for the calling thread.
void set_last_error(const char* msg);
// Status of the launches just issued: FITQ_OK, or FITQ_ERR_CUDA with the CUDA
// error kept for the calling thread, so that the message the entry point
// writes names it (reading cudaGetLastError() clears it).
int launch_result();
// Makes the primary context of the runtime's current device current on the
// calling host thread.  A thread that has not yet made a CUDA runtime call
// that binds one (PyTorch's autograd worker for device 0, a foreign caller's
// own thread) has no current context; launches through the runtime bind it
// themselves, but driver calls such as cuTensorMapEncodeTiled then fail with
// CUDA_ERROR_INVALID_CONTEXT.  The tensor-map encoders call this on that error
// and retry once.
inline bool bind_primary_context() {
  int dev = 0;
  return cudaGetDevice(&dev) == cudaSuccess && cudaSetDevice(dev) == cudaSuccess;
}
// Extra text for the next failure message of the calling thread (what a
// launcher's host-side set-up rejected, e.g. a tensor map the driver refused).
void note_launch_detail(const char* msg);
// fitq_nf4_gemv with the given scratch in place of a caller workspace (abi.cu).
int nf4_gemv_on_scratch(const fitq_nf4_weight* w, const void* x, int64_t m, const float* lora_a,
                        const float* lora_b, int rank, float scale, const void* bias, void* y,
                        const void* y_add, void* scratch, size_t scratch_bytes,
                        fitq_stream_t stream);
void timing_end(int slot, cudaStream_t st);

// Decoder-layer row / elementwise kernels (layer_ops.cu).
int launch_rmsnorm_fwd(const void* x, const void* w, void* y, int64_t rows, int64_t cols,
                       float eps, cudaStream_t st);
int launch_rmsnorm_bwd(const void* dy, const void* x, const void* w, void* dx, int64_t rows,
                       int64_t cols, float eps, cudaStream_t st);
int launch_rope_append(const void* q, const void* k, const void* v, void* q_out, void* k_cache,
                       void* v_cache, const float* cs, const float* sn, int64_t batch, int t_new,
                       int heads, int kv_heads, int dim, int prefix, int cap, cudaStream_t st,
                       int num_sms);
int launch_rope(const void* t, void* out, const float* cs, const float* sn, int64_t rows,
                int heads, int dim, int64_t seq, int backward, cudaStream_t st, int num_sms);
int launch_swiglu_fwd(const void* g, const void* u, void* act, int64_t n, cudaStream_t st,
                      int num_sms);
int launch_swiglu_bwd(const void* d, const void* g, const void* u, void* dg, void* du, int64_t n,
                      cudaStream_t st, int num_sms);

// Optimizer kernels (optim.cu).
int launch_adamw(float* p, const float* g, float* m, float* v, int64_t n, float lr, float b1,
                 float b2, float eps, float wd, int step, const float* clip, cudaStream_t st);
size_t grad_norm_workspace(int64_t n);
int launch_grad_clip(const float* g, int64_t n, float max_norm, float* norm_out, void* ws,
                     cudaStream_t st);

}  // namespace fitq
