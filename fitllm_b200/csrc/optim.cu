// LoRA optimizer kernels: AdamW with FitLLM's update order
// (ShardOptimizer.step_from_memory, fitllm/optimizer.py:206-231) and the
// global-norm clip coefficient of _clip_lora_accum_grads
// (fitllm/trainer.py:70-88), computed on the device so no host sync is needed.
#include "common.cuh"
#include "kernels.cuh"

namespace fitq {
namespace {

constexpr int kNormThreads = 256;
constexpr int64_t kNormChunk = 1 << 16;  // elements per partial sum

// Each step rounds exactly like the reference's sequence of fp32 tensor ops:
//   m = b1*m + (1-b1)*g ; v = b2*v + ((1-b2)*g)*g
//   mh = m/bc1 ; vh = v/bc2 ; delta = lr*(mh/(sqrt(vh)+eps) + wd*p) ; p -= delta
__global__ void adamw_kernel(float* __restrict__ p, const float* __restrict__ g,
                             float* __restrict__ m, float* __restrict__ v, int64_t n, float lr,
                             float b1, float omb1, float b2, float omb2, float eps, float wd,
                             float bc1, float bc2, const float* __restrict__ clip) {
  const float cc = clip ? clip[1] : 1.0f;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    float gi = g[i];
    if (clip) gi = __fmul_rn(gi, cc);
    const float mi = __fadd_rn(__fmul_rn(b1, m[i]), __fmul_rn(omb1, gi));
    const float vi = __fadd_rn(__fmul_rn(b2, v[i]), __fmul_rn(__fmul_rn(omb2, gi), gi));
    m[i] = mi;
    v[i] = vi;
    const float mh = __fdiv_rn(mi, bc1);
    const float vh = __fdiv_rn(vi, bc2);
    const float pi = p[i];
    const float upd = __fadd_rn(__fdiv_rn(mh, __fadd_rn(__fsqrt_rn(vh), eps)), __fmul_rn(wd, pi));
    p[i] = __fsub_rn(pi, __fmul_rn(lr, upd));
  }
}

// partial[b] = sum over [b*chunk, (b+1)*chunk) of g^2 in fp64, fixed tree order.
__global__ void __launch_bounds__(kNormThreads) sumsq_partial_kernel(const float* __restrict__ g,
                                                                     int64_t n,
                                                                     double* __restrict__ partial) {
  __shared__ double red[kNormThreads];
  const int64_t s = blockIdx.x * kNormChunk;
  const int64_t e = s + kNormChunk < n ? s + kNormChunk : n;
  double acc = 0.0;
  for (int64_t i = s + threadIdx.x; i < e; i += kNormThreads) {
    const double x = g[i];
    acc += x * x;
  }
  red[threadIdx.x] = acc;
  __syncthreads();
  for (int w = kNormThreads / 2; w > 0; w >>= 1) {
    if (threadIdx.x < w) red[threadIdx.x] += red[threadIdx.x + w];
    __syncthreads();
  }
  if (threadIdx.x == 0) partial[blockIdx.x] = red[0];
}

__global__ void clip_finish_kernel(const double* __restrict__ partial, int64_t nparts,
                                   float max_norm, float* __restrict__ out) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  double t = 0.0;
  for (int64_t i = 0; i < nparts; ++i) t += partial[i];
  const double norm = sqrt(t);
  out[0] = static_cast<float>(norm);
  out[1] = (max_norm > 0.f && norm > max_norm) ? static_cast<float>(max_norm / (norm + 1e-6)) : 1.0f;
}

}  // namespace

int launch_adamw(float* p, const float* g, float* m, float* v, int64_t n, float lr, float b1,
                 float b2, float eps, float wd, int step, const float* clip, cudaStream_t st) {
  const double bc1 = 1.0 - pow(static_cast<double>(b1), step);
  const double bc2 = 1.0 - pow(static_cast<double>(b2), step);
  const float omb1 = static_cast<float>(1.0 - static_cast<double>(b1));
  const float omb2 = static_cast<float>(1.0 - static_cast<double>(b2));
  int64_t blocks = (n + 255) / 256;
  if (blocks > 4096) blocks = 4096;
  if (blocks < 1) blocks = 1;
  adamw_kernel<<<static_cast<int>(blocks), 256, 0, st>>>(p, g, m, v, n, lr, b1, omb1, b2, omb2,
                                                         eps, wd, static_cast<float>(bc1),
                                                         static_cast<float>(bc2), clip);
  note_launch();
  return launch_result();
}

size_t grad_norm_workspace(int64_t n) {
  const int64_t parts = (n + kNormChunk - 1) / kNormChunk;
  return static_cast<size_t>(parts > 0 ? parts : 1) * sizeof(double);
}

int launch_grad_clip(const float* g, int64_t n, float max_norm, float* norm_out, void* ws,
                     cudaStream_t st) {
  const int64_t parts = (n + kNormChunk - 1) / kNormChunk;
  double* partial = static_cast<double*>(ws);
  if (parts > 0) {
    sumsq_partial_kernel<<<static_cast<int>(parts), kNormThreads, 0, st>>>(g, n, partial);
    note_launch();
  }
  clip_finish_kernel<<<1, 32, 0, st>>>(partial, parts, max_norm, norm_out);
  note_launch();
  return launch_result();
}

}  // namespace fitq
