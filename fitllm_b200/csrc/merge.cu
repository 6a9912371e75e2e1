// LoRA merge into a dense weight: W[n, k] <- W[n, k] + scale * (B . A)[n, k]
// (fitllm/inference.py:127-131, merge_lora_into_shards: W.float() +
// scale * (B @ A), cast back to the weight's dtype), in place on the device.
//
// Each element: t = sum_j B[n, j] * A[j, k] in fp32, j ascending, each
// product and partial sum rounded (no fused multiply-add), then
// fl(float(W) + fl(scale * t)) rounded to the weight's dtype (round to
// nearest even).  HBM-bound: 2 + 2 bytes per weight (4 + 4 for fp32); A and
// B stay in L1/L2.
//
// A CTA of 256 threads owns 16 rows x 512 columns: thread c holds columns
// 2c, 2c+1 and walks the 16 rows with A's two columns in registers 16 ranks
// at a time and B's rows broadcast from shared memory.
#include "common.cuh"
#include "kernels.cuh"

namespace fitq {
namespace {

constexpr int kMergeRows = 16;
constexpr int kMergeCols = 512;
constexpr int kMergeThreads = 256;
constexpr int kMergeRankChunk = 16;

template <typename T>
__device__ __forceinline__ float2 load2(const T* p);
template <>
__device__ __forceinline__ float2 load2<__nv_bfloat16>(const __nv_bfloat16* p) {
  return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(p));
}
template <>
__device__ __forceinline__ float2 load2<__half>(const __half* p) {
  return __half22float2(*reinterpret_cast<const __half2*>(p));
}
template <>
__device__ __forceinline__ float2 load2<float>(const float* p) {
  return *reinterpret_cast<const float2*>(p);
}
template <typename T>
__device__ __forceinline__ void store2(T* p, float a, float b);
template <>
__device__ __forceinline__ void store2<float>(float* p, float a, float b) {
  *reinterpret_cast<float2*>(p) = make_float2(a, b);
}
template <>
__device__ __forceinline__ void store2<__nv_bfloat16>(__nv_bfloat16* p, float a, float b) {
  *reinterpret_cast<__nv_bfloat162*>(p) = __floats2bfloat162_rn(a, b);
}
template <>
__device__ __forceinline__ void store2<__half>(__half* p, float a, float b) {
  *reinterpret_cast<__half2*>(p) = __floats2half2_rn(a, b);
}

template <typename T>
__global__ void __launch_bounds__(kMergeThreads)
    lora_merge_kernel(T* __restrict__ w, int N, int K, const float* __restrict__ a,
                      const float* __restrict__ b, int rank, float scale) {
  extern __shared__ float s_b[];  // [kMergeRows][rank]
  const int n0 = blockIdx.y * kMergeRows;
  const int rows = N - n0 < kMergeRows ? N - n0 : kMergeRows;
  for (int i = threadIdx.x; i < rows * rank; i += kMergeThreads)
    s_b[i] = __ldg(b + static_cast<int64_t>(n0) * rank + i);
  __syncthreads();
  const int k = blockIdx.x * kMergeCols + 2 * threadIdx.x;
  if (k >= K) return;  // K is even: both columns in range
  float t0[kMergeRows], t1[kMergeRows];
#pragma unroll
  for (int r = 0; r < kMergeRows; ++r) t0[r] = t1[r] = 0.f;
  for (int j0 = 0; j0 < rank; j0 += kMergeRankChunk) {
    const int jn = rank - j0 < kMergeRankChunk ? rank - j0 : kMergeRankChunk;
    float2 av[kMergeRankChunk];
#pragma unroll
    for (int j = 0; j < kMergeRankChunk; ++j)
      av[j] = j < jn ? __ldg(reinterpret_cast<const float2*>(a + static_cast<int64_t>(j0 + j) * K + k))
                     : make_float2(0.f, 0.f);
#pragma unroll
    for (int r = 0; r < kMergeRows; ++r) {
      if (r >= rows) break;
      const float* br = s_b + r * rank + j0;
#pragma unroll
      for (int j = 0; j < kMergeRankChunk; ++j) {
        if (j >= jn) break;
        t0[r] = __fadd_rn(t0[r], __fmul_rn(br[j], av[j].x));
        t1[r] = __fadd_rn(t1[r], __fmul_rn(br[j], av[j].y));
      }
    }
  }
#pragma unroll
  for (int r = 0; r < kMergeRows; ++r) {
    if (r >= rows) break;
    T* p = w + static_cast<int64_t>(n0 + r) * K + k;
    const float2 v = load2<T>(p);
    store2<T>(p, __fadd_rn(v.x, __fmul_rn(scale, t0[r])), __fadd_rn(v.y, __fmul_rn(scale, t1[r])));
  }
}

}  // namespace

int launch_lora_merge(void* w, int out_dtype, int64_t n, int64_t k, const float* a, const float* b,
                      int rank, float scale, cudaStream_t st) {
  if (n <= 0 || k <= 0 || (k & 1) || rank <= 0 || rank > 256 || n >= (1ll << 31) ||
      k >= (1ll << 31))
    return FITQ_ERR_SHAPE;
  const dim3 grid(static_cast<unsigned>((k + kMergeCols - 1) / kMergeCols),
                  static_cast<unsigned>((n + kMergeRows - 1) / kMergeRows));
  if (grid.y > 65535u) return FITQ_ERR_SHAPE;
  const size_t smem = static_cast<size_t>(kMergeRows) * rank * sizeof(float);
  const int N = static_cast<int>(n), K = static_cast<int>(k);
  if (out_dtype == FITQ_DTYPE_BF16)
    lora_merge_kernel<__nv_bfloat16><<<grid, kMergeThreads, smem, st>>>(
        static_cast<__nv_bfloat16*>(w), N, K, a, b, rank, scale);
  else if (out_dtype == FITQ_DTYPE_F16)
    lora_merge_kernel<__half><<<grid, kMergeThreads, smem, st>>>(static_cast<__half*>(w), N, K, a,
                                                                  b, rank, scale);
  else
    lora_merge_kernel<float><<<grid, kMergeThreads, smem, st>>>(static_cast<float*>(w), N, K, a, b,
                                                                 rank, scale);
  note_launch();
  return launch_result();
}

}  // namespace fitq
