// Cross-entropy over lm_head logits, forward and backward in one pass per row.
//
// FitLLM computes the loss of every micro-batch as CrossEntropyLoss (mean over
// labels != -100) of the lm_head logits and back-propagates loss * loss_scale
// (fitllm/backward.py:188-198; the logged loss, fitllm/trainer.py:506-522, is
// the same mean on fp32 logits).  Here the logits of one micro-batch ([T, V]
// bf16, written by the tcgen05 GEMM) are turned in place into
// d(loss_scale * loss)/dlogits, and the mean loss is written to a device
// scalar:
//
//   ce_count_kernel   n_valid = #(labels != ignore_index)             (1 CTA)
//   ce_row_kernel     one CTA per row: online max / sum of exp over the row
//                     (16-byte loads, fp32), lse = m + log(s),
//                     loss_t = lse - z[label]; then the same row is rewritten
//                     as (exp(z - lse) - [v == label]) * loss_scale / n_valid
//                     (zeros for an ignored row)
//   ce_finish_kernel  loss = sum_t loss_t / n_valid in row order    (1 CTA)
//
// The row (2 V bytes, 304 KB at V = 152,064) is read twice and written once;
// the second read hits L2.  Deterministic: fixed reduction orders.
#include "common.cuh"
#include "kernels.cuh"

namespace fitq {
namespace {

// 1024 threads: two CTAs (rows) per SM keep ~300 rows in flight, 90 MB at
// V = 152,064, so the second read of a row still finds it in L2 (at four rows
// per SM a third of the second reads went to DRAM).
constexpr int kCeThreads = 1024;

__device__ __forceinline__ void block_reduce_max_sum(float& m, float& s, float* sh_m, float* sh_s) {
  // warp: combine (m, s) pairs
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
    const float s2 = __shfl_xor_sync(0xffffffffu, s, o);
    const float mn = fmaxf(m, m2);
    s = (m == -INFINITY ? 0.f : s * __expf(m - mn)) + (m2 == -INFINITY ? 0.f : s2 * __expf(m2 - mn));
    m = mn;
  }
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) {
    sh_m[w] = m;
    sh_s[w] = s;
  }
  __syncthreads();
  if (w == 0) {
    m = l < kCeThreads / 32 ? sh_m[l] : -INFINITY;
    s = l < kCeThreads / 32 ? sh_s[l] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
      const float s2 = __shfl_xor_sync(0xffffffffu, s, o);
      const float mn = fmaxf(m, m2);
      s = (m == -INFINITY ? 0.f : s * __expf(m - mn)) + (m2 == -INFINITY ? 0.f : s2 * __expf(m2 - mn));
      m = mn;
    }
    if (l == 0) {
      sh_m[0] = m;
      sh_s[0] = s;
    }
  }
  __syncthreads();
  m = sh_m[0];
  s = sh_s[0];
}

__global__ void __launch_bounds__(1024) ce_count_kernel(const int64_t* __restrict__ labels, int64_t T,
                                                         int64_t ignore_index, int* n_valid) {
  __shared__ int sh[32];
  int c = 0;
  for (int64_t i = threadIdx.x; i < T; i += blockDim.x) c += labels[i] != ignore_index ? 1 : 0;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) c += __shfl_xor_sync(0xffffffffu, c, o);
  if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = c;
  __syncthreads();
  if (threadIdx.x == 0) {
    int t = 0;
    for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) t += sh[w];
    *n_valid = t;
  }
}

__global__ void __launch_bounds__(kCeThreads)
    ce_row_kernel(__nv_bfloat16* __restrict__ logits, const int64_t* __restrict__ labels, int64_t V,
                  int64_t ignore_index, float loss_scale, const int* __restrict__ n_valid,
                  float* __restrict__ loss_rows) {
  __shared__ float sh_m[kCeThreads / 32], sh_s[kCeThreads / 32];
  const int64_t t = blockIdx.x;
  uint4* row = reinterpret_cast<uint4*>(logits + t * V);
  const int64_t nv = V / 8;  // V % 8 == 0 (host check)
  float m = -INFINITY, s = 0.f;
  for (int64_t i = threadIdx.x; i < nv; i += kCeThreads) {
    const uint4 u = row[i];
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
    float x[8];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = unpack_bf16x2(w[j]);
      x[2 * j] = f.x;
      x[2 * j + 1] = f.y;
    }
    float vm = x[0];
#pragma unroll
    for (int j = 1; j < 8; ++j) vm = fmaxf(vm, x[j]);
    if (vm > m) {
      s = m == -INFINITY ? 0.f : s * __expf(m - vm);
      m = vm;
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) s += __expf(x[j] - m);
  }
  block_reduce_max_sum(m, s, sh_m, sh_s);
  const float lse = m + __logf(s);
  const int64_t label = labels[t];
  const bool valid = label != ignore_index && label >= 0 && label < V;
  if (threadIdx.x == 0)
    loss_rows[t] = valid ? lse - __bfloat162float(logits[t * V + label]) : 0.f;
  __syncthreads();  // the target logit is read before the row is overwritten
  const int nvalid = *n_valid;
  const float g = (valid && nvalid > 0) ? loss_scale / static_cast<float>(nvalid) : 0.f;
  for (int64_t i = threadIdx.x; i < nv; i += kCeThreads) {
    const uint4 u = row[i];
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
    uint32_t o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = unpack_bf16x2(w[j]);
      const int64_t v0 = 8 * i + 2 * j;
      const float d0 = (__expf(f.x - lse) - (v0 == label ? 1.f : 0.f)) * g;
      const float d1 = (__expf(f.y - lse) - (v0 + 1 == label ? 1.f : 0.f)) * g;
      o[j] = pack_bf16x2(d0, d1);
    }
    row[i] = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

__global__ void __launch_bounds__(1024) ce_finish_kernel(const float* __restrict__ loss_rows, int64_t T,
                                                          const int* __restrict__ n_valid,
                                                          float* __restrict__ loss_out) {
  __shared__ float sh[32];
  float a = 0.f;
  for (int64_t i = threadIdx.x; i < T; i += blockDim.x) a += loss_rows[i];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
  if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = a;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) t += sh[w];
    const int n = *n_valid;
    *loss_out = n > 0 ? t / static_cast<float>(n) : 0.f;
  }
}

}  // namespace

size_t cross_entropy_workspace(int64_t rows) {
  return static_cast<size_t>((rows + 4) * sizeof(float) + 256);
}

int launch_cross_entropy(void* logits, const int64_t* labels, int64_t T, int64_t V,
                         int64_t ignore_index, float loss_scale, float* loss_out, void* workspace,
                         cudaStream_t st) {
  int* n_valid = static_cast<int*>(workspace);
  float* loss_rows = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + 256);
  ce_count_kernel<<<1, 1024, 0, st>>>(labels, T, ignore_index, n_valid);
  note_launch();
  ce_row_kernel<<<static_cast<unsigned>(T), kCeThreads, 0, st>>>(
      static_cast<__nv_bfloat16*>(logits), labels, V, ignore_index, loss_scale, n_valid, loss_rows);
  note_launch();
  ce_finish_kernel<<<1, 1024, 0, st>>>(loss_rows, T, n_valid, loss_out);
  note_launch();
  return launch_result();
}

}  // namespace fitq
