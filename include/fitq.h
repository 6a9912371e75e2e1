/*
 * fitq -- C ABI of the B200 (sm_100a) NF4 QLoRA linear.
 *
 * Every pointer is a device pointer owned by the caller unless stated
 * otherwise; every call is asynchronous on the given stream and returns a
 * status code (FITQ_OK = 0).  No entry point allocates device memory except
 * where a caller-provided workspace is named; no entry point synchronises the
 * stream except fitq_get_device_status.  Shapes that a kernel does not
 * support return an error: there is no fallback path.
 *
 * Reference interfaces these calls replace (paths inside FitLLM; the NF4 and
 * LoRA arithmetic itself lives in bitsandbytes and PEFT, which FitLLM calls):
 *   fitq_nf4_dequant   bitsandbytes dequantize_4bit, run inside every
 *                      bnb.nn.Linear4bit forward (fitllm/forward.py:511 ->
 *                      _run_layer, fitllm/forward.py:680-686) and again in
 *                      MatMul4Bit.backward (fitllm/backward.py:234).
 *   fitq_nf4_quantize  bitsandbytes quantize_4bit(nf4, compress_statistics)
 *                      run at load time by BitsAndBytesConfig
 *                      (fitllm/model.py:211-219).
 *   fitq_qlora_fwd     PEFT lora.Linear4bit.forward = Linear4bit.forward +
 *                      lora_B(lora_A(x)) * scaling (fitllm/qlora.py:74-83),
 *                      entered from fitllm/forward.py:511 and the recompute
 *                      in fitllm/backward.py:222-231.
 *   fitq_qlora_bwd     autograd of the above: MatMul4Bit.backward (dX through
 *                      the dequantised weight) + the LoRA graph (dA, dB),
 *                      entered by h_out.backward (fitllm/backward.py:234);
 *                      grad_accumulate mirrors _accumulate_grads_to_ram
 *                      (fitllm/backward.py:287-299).
 *   fitq_nf4_gemv      bitsandbytes gemv_4bit, the single-token decode path of
 *                      matmul_4bit (fitllm/forward.py:623-625), widened to the
 *                      speculative-verify row counts (M <= 64,
 *                      fitllm/inference.py:380-397).
 *   fitq_adamw_step    ShardOptimizer.step_from_memory AdamW update
 *                      (fitllm/optimizer.py:161-231) with the global-norm clip
 *                      of _clip_lora_accum_grads (fitllm/trainer.py:70-88).
 *   fitq_gemm_bf16_tn  (building block, no direct reference counterpart) the
 *                      tcgen05 GEMM that the fused paths are built on.
 */
#ifndef FITQ_H
#define FITQ_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define FITQ_API __attribute__((visibility("default")))
#else
#define FITQ_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

enum {
  FITQ_OK = 0,
  FITQ_ERR_ARG = 1,         /* null pointer or invalid scalar argument       */
  FITQ_ERR_SHAPE = 2,       /* a dimension the kernels do not support        */
  FITQ_ERR_ALIGN = 3,       /* a pointer or row pitch not 16-byte aligned    */
  FITQ_ERR_UNSUPPORTED = 4, /* valid request outside the implemented range   */
  FITQ_ERR_WORKSPACE = 5,   /* workspace missing or smaller than required    */
  FITQ_ERR_CUDA = 6,        /* CUDA runtime / driver call failed             */
  FITQ_ERR_TIMEOUT = 7,     /* a bounded device-side wait ran out            */
  FITQ_ERR_NO_DEVICE = 8    /* no usable sm_100 device                       */
};

/* A cudaStream_t (CUstream) handle; NULL is the legacy default stream.
 * Every call is asynchronous on the given stream.  fitq_qlora_fwd and
 * fitq_qlora_bwd on the GEMM path (M > 64) fork the weight-side launches
 * (NF4 dequant, LoRA weight padding) onto one internal stream per device and
 * join it back before returning, with events, so a call captured into a CUDA
 * graph captures the fork too; set FITQ_SIDE_STREAM=0 in the environment to
 * keep every launch on the given stream.  The internal stream is shared by
 * the process's calls on that device: a stream capture on one host thread
 * must not overlap uncaptured GEMM-path calls on the same device from
 * another thread. */
typedef void* fitq_stream_t;

/* One NF4 weight W[N,K] in the bitsandbytes Params4bit layout (flat keys
 * <param>, .absmax, .nested_absmax, .quant_map, .nested_quant_map and the
 * nested_offset of .quant_state.bitsandbytes__nf4, fitllm/forward.py:95-109).
 * packed: N*K/2 bytes, flat row-major, element 2i in the high nibble.
 * Double-quantised statistics: absmax_code (one uint8 per 64 elements),
 * nested_absmax (one fp32 per 256 codes), nested_quant_map (256 fp32), offset.
 * A state without double quantisation sets absmax_f32 (one fp32 per 64
 * elements) instead and leaves the three nested fields NULL. */
typedef struct fitq_nf4_weight {
  const uint8_t* packed;
  const uint8_t* absmax_code;
  const float* nested_absmax;
  const float* nested_quant_map;
  const float* absmax_f32;
  const float* quant_map;
  float offset;
  int64_t n_out;
  int64_t k_in;
} fitq_nf4_weight;

/* Output dtypes of fitq_nf4_dequant (bf16, fp16) and weight dtypes of
 * fitq_lora_merge (all three). */
enum { FITQ_DTYPE_BF16 = 0, FITQ_DTYPE_F16 = 1, FITQ_DTYPE_F32 = 2 };

FITQ_API const char* fitq_version(void);

/* Text of the last host-side error seen by this thread (never NULL). */
FITQ_API const char* fitq_last_error(void);

/* Synchronise `stream`, then return the device status word (FITQ_OK or the
 * first FITQ_ERR_* a kernel recorded, e.g. FITQ_ERR_TIMEOUT).  reset != 0
 * clears it afterwards. */
FITQ_API int fitq_get_device_status(int reset, fitq_stream_t stream);

/* Self-test of the failure path of the device waits (no fault involved): one
 * thread waits, with the bounded mbarrier wait every pipelined kernel uses,
 * on a barrier that nothing completes; after limit_ns (1 us .. 1 s) it records
 * FITQ_ERR_TIMEOUT in the device status word and the kernel returns, leaving
 * the context usable.  elapsed_ns (device, optional) receives the time waited.
 * Returns FITQ_OK once launched; read the outcome with fitq_get_device_status. */
FITQ_API int fitq_selftest_wait_timeout(uint64_t limit_ns, unsigned long long* elapsed_ns,
                                        fitq_stream_t stream);

/* W -> out, bit-exact: absmax_b = fl(fl(nqm[code_b]*nabs[b/256]) + offset),
 * w = fl(qm[nibble]*absmax_b) rounded to nearest even into bf16 or fp16.
 * transpose = 0 writes out[N,K]; transpose = 1 writes out[K,N].
 * Requires K % 64 == 0 and, for transpose, N % 64 == 0. */
FITQ_API int fitq_nf4_dequant(const fitq_nf4_weight* w, void* out, int out_dtype, int transpose,
                     fitq_stream_t stream);

/* fp32 W[N,K] -> NF4 with double-quantised absmax.  quant_map (16) and
 * nested_quant_map (256) are the sorted level tables to use; offset_out
 * receives the fp32 mean of the first-level absmax (device, 1 float).
 * workspace >= fitq_nf4_quantize_workspace(N, K) bytes. */
FITQ_API size_t fitq_nf4_quantize_workspace(int64_t n_out, int64_t k_in);
FITQ_API int fitq_nf4_quantize(const float* w, int64_t n_out, int64_t k_in, const float* quant_map,
                      const float* nested_quant_map, uint8_t* packed, uint8_t* absmax_code,
                      float* nested_absmax, float* offset_out, void* workspace,
                      size_t workspace_bytes, fitq_stream_t stream);

/* y[M,N] (bf16) = x[M,K].W^T + scale.(x.A^T).B^T (+ bias[N]) (+ y_add[M,N]).
 * x bf16 row-major; lora_a fp32 [rank,K] and lora_b fp32 [N,rank] (PEFT
 * layout), both NULL (rank 0) for a bare Linear4bit; bias bf16 [N] or NULL
 * (Linear4bit's frozen bias); y_add bf16 [M,N] or NULL (fused residual).  t_out, if non-NULL,
 * receives T = x.A^T as bf16 [M,rank] for the backward.  rank in {0,16,32,48,64};
 * lora_b 16-byte aligned.  M <= 64 runs the NF4 GEMV kernels (M <= 8: one
 * launch, plus a LoRA and a finishing launch that overlap it when needed),
 * larger M the tcgen05 GEMM. */
FITQ_API size_t fitq_qlora_fwd_workspace(int64_t m, int64_t n_out, int64_t k_in, int rank);
FITQ_API int fitq_qlora_fwd(const fitq_nf4_weight* w, const void* x, int64_t m, const float* lora_a,
                   const float* lora_b, int rank, float scale, const void* bias, void* y,
                   const void* y_add, void* t_out, void* workspace, size_t workspace_bytes,
                   fitq_stream_t stream);

/* Backward of fitq_qlora_fwd for upstream grad dy[M,N] (bf16):
 *   dx[M,K]       = dy.W + scale.(dy.B).A            (bf16; += if dx_accumulate)
 *   grad_a[rank,K] = scale.(dy.B)^T.x                 (fp32; += if grad_accumulate)
 *   grad_b[N,rank] = scale.dy^T.(x.A^T)               (fp32; += if grad_accumulate)
 * t_saved: T from the forward (bf16 [M,rank]) or NULL to recompute it.
 * dx may be NULL (no input grad); grad_a/grad_b NULL when rank == 0. */
FITQ_API size_t fitq_qlora_bwd_workspace(int64_t m, int64_t n_out, int64_t k_in, int rank);
FITQ_API int fitq_qlora_bwd(const fitq_nf4_weight* w, const void* x, const void* dy, int64_t m,
                   const float* lora_a, const float* lora_b, int rank, float scale,
                   const void* t_saved, void* dx, int dx_accumulate, float* grad_a,
                   float* grad_b, int grad_accumulate, void* workspace, size_t workspace_bytes,
                   fitq_stream_t stream);

/* Decode / speculative-verify projection for M <= 64 rows: the NF4 weight is
 * streamed once from HBM and decoded on the fly into tensor-core operands.
 * Same arithmetic contract as fitq_qlora_fwd; needs N % 64 == 0 and
 * K % 256 == 0 (fitq_qlora_fwd uses it for such shapes when M <= 64). */
FITQ_API size_t fitq_nf4_gemv_workspace(int64_t m, int64_t n_out, int64_t k_in, int rank);
FITQ_API int fitq_nf4_gemv(const fitq_nf4_weight* w, const void* x, int64_t m, const float* lora_a,
                  const float* lora_b, int rank, float scale, const void* bias, void* y,
                  const void* y_add, void* workspace, size_t workspace_bytes,
                  fitq_stream_t stream);

/* One projection of a grouped GEMV: y[M, N] = x.W^T + scale.(x.A^T).B^T
 * (+ bias) (+ y_add), the fitq_nf4_gemv arguments of one weight. */
typedef struct fitq_gemv_job {
  const fitq_nf4_weight* w;
  const float* lora_a; /* fp32 [rank, K] or NULL */
  const float* lora_b; /* fp32 [N, rank] or NULL */
  int rank;
  float scale;
  const void* bias;    /* bf16 [N] or NULL */
  void* y;             /* bf16 [M, N] */
  const void* y_add;   /* bf16 [M, N] or NULL */
} fitq_gemv_job;

/* Up to three projections of the same x (q/k/v, gate/up of a decoder layer:
 * the HF layer runs them as separate Linear4bit calls, fitllm/forward.py:
 * 680-686), each with fitq_nf4_gemv's result.  For 8 < M <= 64 with a shared
 * K and scale format they run as ONE tcgen05 launch over all their tiles
 * (small projections such as k/v no longer split K many ways on their own);
 * otherwise one fitq_nf4_gemv per job, in order. */
FITQ_API size_t fitq_nf4_gemv_grouped_workspace(const fitq_gemv_job* jobs, int count, int64_t m);
FITQ_API int fitq_nf4_gemv_grouped(const fitq_gemv_job* jobs, int count, const void* x, int64_t m,
                                   void* workspace, size_t workspace_bytes, fitq_stream_t stream);

/* The MLP input of a decoder layer: act[M, N] = SiLU(gate) * up with
 * gate = x.Wg^T, up = x.Wu^T (jobs[0], jobs[1]; rank 0, same shape; their y
 * is not written), the HF Qwen2MLP's act_fn(gate_proj(x)) * up_proj(x) that
 * fitllm/forward.py:680-686 runs per layer.  Bit-identical to
 * fitq_nf4_gemv_grouped followed by fitq_swiglu_fwd; on the grouped tcgen05
 * path the SwiGLU is applied in the finishing pass, so gate and up are never
 * stored. */
FITQ_API size_t fitq_nf4_gemv_swiglu_workspace(const fitq_gemv_job* jobs, int64_t m);
FITQ_API int fitq_nf4_gemv_swiglu(const fitq_gemv_job* jobs, const void* x, int64_t m, void* act,
                                  void* workspace, size_t workspace_bytes, fitq_stream_t stream);

/* c[M,N] (bf16) = a[M,K].b[N,K]^T (+ c_add) on the tcgen05 tensor cores,
 * fp32 accumulation.  K % 64 == 0, N % 16 == 0, rows 16-byte aligned. */
FITQ_API int fitq_gemm_bf16_tn(const void* a, const void* b, void* c, const void* c_add, int64_t m,
                      int64_t n, int64_t k, fitq_stream_t stream);

/* AdamW over n fp32 values, in place on param/exp_avg/exp_avg_sq:
 *   g = grad * clip;  m = b1 m + (1-b1) g;  v = b2 v + (1-b2) g^2
 *   param -= lr * (m/(1-b1^t) / (sqrt(v/(1-b2^t)) + eps) + wd * param)
 * clip: device fp32 scalar from fitq_grad_clip_coef, or NULL for 1. */
FITQ_API int fitq_adamw_step(float* param, const float* grad, float* exp_avg, float* exp_avg_sq,
                    int64_t n, float lr, float beta1, float beta2, float eps,
                    float weight_decay, int step, const float* clip, fitq_stream_t stream);

/* Global L2 norm of n fp32 values (all LoRA grads of a step, one flat
 * buffer) -> norm_out[0], and the clip coefficient -> norm_out[1]:
 * max_norm/(norm+1e-6) when max_norm > 0 and norm > max_norm, else 1
 * (_clip_lora_accum_grads, fitllm/trainer.py:70-88).  Deterministic (fixed
 * fp64 summation order).  workspace >= fitq_grad_norm_workspace(n) bytes. */
FITQ_API size_t fitq_grad_norm_workspace(int64_t n);
FITQ_API int fitq_grad_clip_coef(const float* grads, int64_t n, float max_norm, float* norm_out,
                        void* workspace, size_t workspace_bytes, fitq_stream_t stream);

/* Launch timing of the tcgen05 GEMM kernel (measurement aid, host-side only):
 * fitq_timing_enable(capacity) starts recording a CUDA event pair on the
 * launching stream around each GEMM launch (up to `capacity` launches; 0
 * stops).  fitq_timing_read waits for the recorded events and writes, per
 * launch, the device time in ms and the launch's algorithmic FLOPs
 * (2.M.N.(K + lora_k)); it returns the number of launches (<= max). */
FITQ_API int fitq_timing_enable(int capacity);
FITQ_API int fitq_timing_read(float* ms, double* flops, int max);

/* Decoder-layer kernels around the projections (HF Qwen2DecoderLayer as
 * FitLLM runs it, fitllm/forward.py:657-701; torch ops in the reference).
 * bf16 tensors, fp32 arithmetic, one pass each.
 * RMSNorm (Qwen2RMSNorm): y = w * bf16(x * rsqrt(mean(x^2) + eps)) per row of
 * `cols` (cols % 8 == 0); the backward returns dx only (w is frozen).
 * Rotary embedding (rotate-half) on t[rows, heads, head_dim], position =
 * row % seq, cos_half/sin_half fp32 [seq, head_dim/2]; backward != 0 applies
 * the transposed rotation (the gradient).  head_dim % 16 == 0.
 * SwiGLU: act = silu(gate) * up over n elements (n % 8 == 0) and its
 * gradients d_gate, d_up. */
FITQ_API int fitq_rmsnorm_fwd(const void* x, const void* weight, void* y, int64_t rows,
                              int64_t cols, float eps, fitq_stream_t stream);
FITQ_API int fitq_rmsnorm_bwd(const void* dy, const void* x, const void* weight, void* dx,
                              int64_t rows, int64_t cols, float eps, fitq_stream_t stream);
FITQ_API int fitq_rope(const void* t, void* out, const float* cos_half, const float* sin_half,
                       int64_t rows, int heads, int head_dim, int64_t seq, int backward,
                       fitq_stream_t stream);
FITQ_API int fitq_swiglu_fwd(const void* gate, const void* up, void* act, int64_t n,
                             fitq_stream_t stream);

/* Verify step with a KV cache: rotary embedding of the T new tokens' q and k
 * (positions prefix + t, fp32 half tables cos/sin [T, head_dim/2], the
 * fitq_rope arithmetic) and the append of rotated k and of v to the caches
 * [B, KVH, capacity, head_dim] at [prefix, prefix + T), one launch.
 * q, q_out: [B*T, heads*head_dim]; k, v: [B*T, kv_heads*head_dim] bf16. */
FITQ_API int fitq_rope_append(const void* q, const void* k, const void* v, void* q_out,
                              void* k_cache, void* v_cache, const float* cos_half,
                              const float* sin_half, int64_t batch, int t_new, int heads,
                              int kv_heads, int head_dim, int prefix, int capacity,
                              fitq_stream_t stream);

/* Cross-entropy of lm_head logits, forward and backward: loss_out (device
 * fp32 scalar) = mean over rows with label != ignore_index of
 * logsumexp(logits[t]) - logits[t, label[t]] (torch CrossEntropyLoss, as
 * FitLLM applies it per micro-batch: fitllm/backward.py:188-198), and logits
 * [rows, vocab] bf16 are OVERWRITTEN with d(loss_scale * loss)/dlogits.
 * labels: int64 [rows]; labels outside [0, vocab) other than ignore_index
 * contribute nothing.  vocab % 8 == 0. */
FITQ_API size_t fitq_cross_entropy_workspace(int64_t rows);
FITQ_API int fitq_cross_entropy(void* logits, const int64_t* labels, int64_t rows, int64_t vocab,
                                int64_t ignore_index, float loss_scale, float* loss_out,
                                void* workspace, size_t workspace_bytes, fitq_stream_t stream);

/* Speculative-verify attention over a key/value cache.  Replaces the
 * re-run of the whole prefix that verifies draft tokens (fitllm/inference.py:
 * 380-397, attention inside fitllm/forward.py's layer forward): the T new
 * tokens of each sequence attend to prefix + T cached positions, token i to
 * positions <= prefix + i.  q, out: [B, T, H, head_dim] bf16 (post-RoPE q_proj
 * output / o_proj input); k_cache, v_cache: [B, KVH, capacity, head_dim] bf16
 * with the new tokens' keys/values already at [prefix, prefix + T).  Scale
 * 1/sqrt(head_dim), fp32 softmax and accumulation.  Needs head_dim == 128 and
 * (H / KVH) * T <= 32 (FITQ_ERR_UNSUPPORTED otherwise). */
FITQ_API size_t fitq_verify_attention_workspace(int64_t batch, int heads, int kv_heads, int t_new,
                                                int prefix);
FITQ_API int fitq_verify_attention(const void* q, const void* k_cache, const void* v_cache,
                                   void* out, int64_t batch, int heads, int kv_heads, int t_new,
                                   int prefix, int capacity, int head_dim, void* workspace,
                                   size_t workspace_bytes, fitq_stream_t stream);

/* Causal grouped-query attention of the training layer, forward and
 * backward.  Replaces the attention of the Qwen2 decoder layer FitLLM runs in
 * the shard-stationary forward and in the backward's recompute (HF layer via
 * fitllm/forward.py:657-701, fitllm/backward.py:222-231):
 * O = softmax(Q K^T / sqrt(head_dim) + causal mask) V, query head h reading
 * KV head h / (heads / kv_heads).
 *   q, o, d_o, dq: [batch, seq, heads, head_dim] bf16 (the q_proj output /
 *                  o_proj input, row-major, no transposes);
 *   k, v, dk, dv:  [batch, seq, kv_heads, head_dim] bf16;
 *   lse:           [batch, heads, seq] fp32, written by the forward and read
 *                  by the backward (the row's log-sum-exp of the scaled
 *                  scores, in base-2 units);
 *   workspace:     fitq_attention_bwd_workspace bytes (fp32 row sums of
 *                  dO . O).
 * fp32 softmax and accumulation; P and dS enter the tensor cores as bf16.
 * The backward is deterministic (no atomics).  Needs head_dim == 128
 * (FITQ_ERR_UNSUPPORTED otherwise), seq % 64 == 0 and heads % kv_heads == 0
 * (FITQ_ERR_SHAPE), 16-byte aligned pointers (FITQ_ERR_ALIGN). */
FITQ_API int fitq_attention_fwd(const void* q, const void* k, const void* v, void* o, float* lse,
                                int64_t batch, int64_t seq, int heads, int kv_heads, int head_dim,
                                fitq_stream_t stream);
FITQ_API size_t fitq_attention_bwd_workspace(int64_t batch, int64_t seq, int heads);
FITQ_API int fitq_attention_bwd(const void* q, const void* k, const void* v, const void* o,
                                const void* d_o, const float* lse, void* dq, void* dk, void* dv,
                                int64_t batch, int64_t seq, int heads, int kv_heads, int head_dim,
                                void* workspace, size_t workspace_bytes, fitq_stream_t stream);
FITQ_API int fitq_swiglu_bwd(const void* d_act, const void* gate, const void* up, void* d_gate,
                             void* d_up, int64_t n, fitq_stream_t stream);

/* The MLP input of a Qwen2 decoder layer, act_fn(gate_proj(x)) * up_proj(x)
 * (HF Qwen2MLP as FitLLM runs it, fitllm/forward.py:680-686), as ONE tcgen05
 * GEMM over both NF4 weights: each output tile holds matching gate and up
 * columns and the epilogue stores act = silu(g) * u of the bf16-rounded
 * products g, u (the arithmetic of fitq_swiglu_fwd, so the result is
 * bit-identical to two fitq_qlora_fwd calls + fitq_swiglu_fwd).  gate_out /
 * up_out (bf16 [m, N], may be NULL) receive g and u for the backward.  The two
 * weights have the same shape [N, K], N % 128 == 0, no bias or LoRA. */
FITQ_API size_t fitq_nf4_gateup_swiglu_workspace(int64_t m, int64_t n_out, int64_t k_in);
FITQ_API int fitq_nf4_gateup_swiglu(const fitq_nf4_weight* w_gate, const fitq_nf4_weight* w_up,
                                    const void* x, int64_t m, void* act, void* gate_out,
                                    void* up_out, void* workspace, size_t workspace_bytes,
                                    fitq_stream_t stream);
/* down_proj's input gradient fused with the SwiGLU backward (the autograd of
 * down_proj(act_fn(gate) * up) at h_out.backward, fitllm/backward.py:234):
 * d_act = dy [m, N] . W_down [N, K] rounded to bf16, then d_gate and d_up
 * (bf16 [m, K]) from the saved gate / up with the arithmetic of
 * fitq_swiglu_bwd -- bit-identical to fitq_qlora_bwd (dX) + fitq_swiglu_bwd;
 * d_act itself is never stored.  No LoRA on down_proj. */
FITQ_API size_t fitq_nf4_down_dswiglu_workspace(int64_t m, int64_t n_out, int64_t k_in);
FITQ_API int fitq_nf4_down_dswiglu(const fitq_nf4_weight* w_down, const void* dy, int64_t m,
                                   const void* gate, const void* up, void* d_gate, void* d_up,
                                   void* workspace, size_t workspace_bytes, fitq_stream_t stream);

/* LoRA merge into a dense weight, in place: W[N,K] <- W + scale * (B . A),
 * the per-weight step of FitLLM's merge_lora_into_shards
 * (fitllm/inference.py:127-131: (W.float() + scale * (B @ A)).to(dtype)).
 * w: bf16, fp16 or fp32 (w_dtype FITQ_DTYPE_BF16 / _F16 / _F32), row-major,
 * 4-byte (fp32: 8-byte) aligned, K even; lora_a fp32 [rank, K] (8-byte aligned), lora_b
 * fp32 [N, rank]; 1 <= rank <= 256.  Per element the rank sum runs in fp32
 * in rank order with every product and sum rounded, then
 * fl(W + fl(scale * sum)) is rounded to w's dtype.  An NF4 weight is merged
 * by dequantising it (fitq_nf4_dequant), merging, and re-quantising
 * (fitq_nf4_quantize). */
FITQ_API int fitq_lora_merge(void* w, int w_dtype, int64_t n_out, int64_t k_in,
                             const float* lora_a, const float* lora_b, int rank, float scale,
                             fitq_stream_t stream);

/* Number of kernels this library has launched in this process so far. */
FITQ_API long long fitq_launch_count(void);

/* fitq_nf4_gemv without a workspace argument, for callers that cannot
 * allocate device memory (no counterpart in the reference: FitLLM always runs
 * with PyTorch's allocator).  Meant for runtimes that drive the decode step
 * through this ABI but own no CUDA allocator, or must account for every
 * device allocation up front: they pass the inputs and outputs they hold, and
 * the scratch comes from one fixed array of FITQ_GEMV_NOALLOC_SCRATCH_BYTES
 * (8 MiB) built into the library, which every GPU that loads the library
 * keeps until the process exits.  Same arguments, checks, kernels and
 * arithmetic as fitq_nf4_gemv (M <= 64, N % 64 == 0, K % 256 == 0, rank
 * 0/16/32/48/64; lora_a, lora_b 16-byte aligned), so the results are
 * bit-identical to it; shapes whose scratch exceeds the array return
 * FITQ_ERR_WORKSPACE with the needed size in fitq_last_error().  The first call on a device looks up the
 * array's device address (cudaGetSymbolAddress) with that device current, so
 * make it before any stream capture.  All calls share the array and each one
 * overwrites what it uses; calls that overlap on the GPU (two streams, two
 * host threads) race on it and must be serialised by the caller. */
#define FITQ_GEMV_NOALLOC_SCRATCH_BYTES ((size_t)8 << 20)
FITQ_API int fitq_nf4_gemv_noalloc(const fitq_nf4_weight* w, const void* x, int64_t m,
                                   const float* lora_a, const float* lora_b, int rank,
                                   float scale, const void* bias, void* y, const void* y_add,
                                   fitq_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* FITQ_H */
