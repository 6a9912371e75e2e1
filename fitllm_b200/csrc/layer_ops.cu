// Fused elementwise / row kernels of the decoder layer around the QLoRA
// projections (HF Qwen2DecoderLayer as FitLLM runs it, fitllm/forward.py:657-701):
// RMSNorm (forward and input-gradient), rotary position embedding on q/k
// (forward and gradient) and the SwiGLU activation silu(gate)*up (forward and
// gradient).  Each is one pass over HBM with 16-byte vector accesses; all
// arithmetic in fp32, bf16 in/out.
#include "common.cuh"
#include "kernels.cuh"

namespace fitq {
namespace {

constexpr int kRowThreads = 256;

__device__ __forceinline__ void load8(const __nv_bfloat16* p, float (&f)[8]) {
  const uint4 v = *reinterpret_cast<const uint4*>(p);
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 t = unpack_bf16x2(w[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}

__device__ __forceinline__ void store8(__nv_bfloat16* p, const float (&f)[8]) {
  uint4 v;
  v.x = pack_bf16x2(f[0], f[1]);
  v.y = pack_bf16x2(f[2], f[3]);
  v.z = pack_bf16x2(f[4], f[5]);
  v.w = pack_bf16x2(f[6], f[7]);
  *reinterpret_cast<uint4*>(p) = v;
}

__device__ __forceinline__ float bf16_round(float x) {
  return __bfloat162float(__float2bfloat16_rn(x));
}

template <int N>
__device__ __forceinline__ void block_sum(float (&v)[N], float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int i = 0; i < N; ++i)
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v[i] += __shfl_xor_sync(0xffffffffu, v[i], o);
  __syncthreads();
  if (lane == 0)
#pragma unroll
    for (int i = 0; i < N; ++i) red[warp * N + i] = v[i];
  __syncthreads();
#pragma unroll
  for (int i = 0; i < N; ++i) {
    float s = 0.f;
    for (int w = 0; w < kRowThreads / 32; ++w) s += red[w * N + i];
    v[i] = s;
  }
}

// y = bf16(w * bf16(x * rsqrt(mean(x^2) + eps)))  (Qwen2RMSNorm rounding points)
__global__ void __launch_bounds__(kRowThreads) rmsnorm_fwd_kernel(
    const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ w,
    __nv_bfloat16* __restrict__ y, int64_t cols, float eps) {
  __shared__ float red[kRowThreads / 32];
  pdl_launch_dependents();
  pdl_wait();  // x comes from the previous kernel
  const int64_t row = blockIdx.x;
  const __nv_bfloat16* xr = x + row * cols;
  float ss[1] = {0.f};
  for (int64_t c = threadIdx.x * 8; c < cols; c += kRowThreads * 8) {
    float f[8];
    load8(xr + c, f);
#pragma unroll
    for (int i = 0; i < 8; ++i) ss[0] = fmaf(f[i], f[i], ss[0]);
  }
  block_sum<1>(ss, red);
  const float r = rsqrtf(ss[0] / static_cast<float>(cols) + eps);
  __nv_bfloat16* yr = y + row * cols;
  for (int64_t c = threadIdx.x * 8; c < cols; c += kRowThreads * 8) {
    float f[8], g[8];
    load8(xr + c, f);
    load8(w + c, g);
#pragma unroll
    for (int i = 0; i < 8; ++i) f[i] = g[i] * bf16_round(f[i] * r);
    store8(yr + c, f);
  }
}

// dx = r*dh - (r^3/D) * x * sum(dh*x),  dh = dy * w   (weight frozen)
__global__ void __launch_bounds__(kRowThreads) rmsnorm_bwd_kernel(
    const __nv_bfloat16* __restrict__ dy, const __nv_bfloat16* __restrict__ x,
    const __nv_bfloat16* __restrict__ w, __nv_bfloat16* __restrict__ dx, int64_t cols,
    float eps) {
  __shared__ float red[2 * kRowThreads / 32];
  const int64_t row = blockIdx.x;
  const __nv_bfloat16* xr = x + row * cols;
  const __nv_bfloat16* dr = dy + row * cols;
  float acc[2] = {0.f, 0.f};  // sum x^2, sum dh*x
  for (int64_t c = threadIdx.x * 8; c < cols; c += kRowThreads * 8) {
    float f[8], d[8], g[8];
    load8(xr + c, f);
    load8(dr + c, d);
    load8(w + c, g);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      acc[0] = fmaf(f[i], f[i], acc[0]);
      acc[1] = fmaf(d[i] * g[i], f[i], acc[1]);
    }
  }
  block_sum<2>(acc, red);
  const float inv_d = 1.0f / static_cast<float>(cols);
  const float r = rsqrtf(acc[0] * inv_d + eps);
  const float k = r * r * r * inv_d * acc[1];
  __nv_bfloat16* out = dx + row * cols;
  for (int64_t c = threadIdx.x * 8; c < cols; c += kRowThreads * 8) {
    float f[8], d[8], g[8];
    load8(xr + c, f);
    load8(dr + c, d);
    load8(w + c, g);
#pragma unroll
    for (int i = 0; i < 8; ++i) f[i] = r * d[i] * g[i] - k * f[i];
    store8(out + c, f);
  }
}

// Rotary embedding on t[rows, heads, D] (rows = batch*seq, position = row % seq),
// rotate-half convention: out[i] = t[i] c_i - t[i+h] s_i, out[i+h] = t[i+h] c_i + t[i] s_i
// (h = D/2).  Gradient: dt[i] = g[i] c_i + g[i+h] s_i, dt[i+h] = g[i+h] c_i - g[i] s_i.
template <bool kBackward>
__global__ void rope_kernel(const __nv_bfloat16* __restrict__ t, __nv_bfloat16* __restrict__ out,
                            const float* __restrict__ cs, const float* __restrict__ sn,
                            int64_t rows, int heads, int dim, int64_t seq) {
  const int half = dim / 2;
  const int groups = half / 8;  // 8-element groups per half
  const int64_t total = rows * heads * groups;
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total;
       e += (int64_t)gridDim.x * blockDim.x) {
    const int gi = static_cast<int>(e % groups);
    const int64_t rh = e / groups;  // row * heads + head
    const int64_t row = rh / heads;
    const int64_t pos = row % seq;
    const int64_t base = rh * dim + gi * 8;
    float a[8], b[8], c[8], s[8];
    load8(t + base, a);
    load8(t + base + half, b);
    const float4* cp = reinterpret_cast<const float4*>(cs + pos * half + gi * 8);
    const float4* sp = reinterpret_cast<const float4*>(sn + pos * half + gi * 8);
    const float4 c0 = cp[0], c1 = cp[1], s0 = sp[0], s1 = sp[1];
    c[0] = c0.x; c[1] = c0.y; c[2] = c0.z; c[3] = c0.w; c[4] = c1.x; c[5] = c1.y; c[6] = c1.z; c[7] = c1.w;
    s[0] = s0.x; s[1] = s0.y; s[2] = s0.z; s[3] = s0.w; s[4] = s1.x; s[5] = s1.y; s[6] = s1.z; s[7] = s1.w;
    float oa[8], ob[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      if (!kBackward) {
        oa[i] = a[i] * c[i] - b[i] * s[i];
        ob[i] = b[i] * c[i] + a[i] * s[i];
      } else {
        oa[i] = a[i] * c[i] + b[i] * s[i];
        ob[i] = b[i] * c[i] - a[i] * s[i];
      }
    }
    store8(out + base, oa);
    store8(out + base + half, ob);
  }
}

// Verify step: rotary embedding of the new tokens' q and k plus the append of
// k (rotated) and v to the KV cache, one launch.  Row b * T + t of q/k/v is
// token t of sequence b at position prefix + t (cos/sin row t); work item =
// (row, head slot, 8-element group of a half), head slots: H of q, KVH of k,
// KVH of v (copied unrotated).  Same arithmetic as rope_kernel<false>.
__global__ void rope_append_kernel(const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ k,
                                   const __nv_bfloat16* __restrict__ v, __nv_bfloat16* __restrict__ q_out,
                                   __nv_bfloat16* __restrict__ kc, __nv_bfloat16* __restrict__ vc,
                                   const float* __restrict__ cs, const float* __restrict__ sn, int64_t rows,
                                   int T, int H, int KVH, int dim, int prefix, int cap) {
  pdl_launch_dependents();
  pdl_wait();  // q/k/v come from the previous kernel
  const int half = dim / 2;
  const int groups = half / 8;
  const int slots = H + 2 * KVH;
  const int64_t total = rows * slots * groups;
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total;
       e += (int64_t)gridDim.x * blockDim.x) {
    const int gi = static_cast<int>(e % groups);
    const int64_t rs = e / groups;
    const int slot = static_cast<int>(rs % slots);
    const int64_t row = rs / slots;
    const int t = static_cast<int>(row % T);
    const int64_t b = row / T;
    const __nv_bfloat16* src;
    __nv_bfloat16* dst;
    if (slot < H) {
      src = q + (row * H + slot) * dim;
      dst = q_out + (row * H + slot) * dim;
    } else {
      const int kh = slot < H + KVH ? slot - H : slot - H - KVH;
      src = (slot < H + KVH ? k : v) + (row * KVH + kh) * dim;
      dst = (slot < H + KVH ? kc : vc) + ((b * KVH + kh) * cap + prefix + t) * static_cast<int64_t>(dim);
    }
    float a[8], bb[8];
    load8(src + gi * 8, a);
    load8(src + half + gi * 8, bb);
    if (slot < H + KVH) {
      const float4* cp = reinterpret_cast<const float4*>(cs + static_cast<int64_t>(t) * half + gi * 8);
      const float4* sp = reinterpret_cast<const float4*>(sn + static_cast<int64_t>(t) * half + gi * 8);
      const float4 c0 = cp[0], c1 = cp[1], s0 = sp[0], s1 = sp[1];
      const float c[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
      const float s[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
      float oa[8], ob[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        oa[i] = a[i] * c[i] - bb[i] * s[i];
        ob[i] = bb[i] * c[i] + a[i] * s[i];
      }
      store8(dst + gi * 8, oa);
      store8(dst + half + gi * 8, ob);
    } else {
      store8(dst + gi * 8, a);
      store8(dst + half + gi * 8, bb);
    }
  }
}


// act = silu(g) * u
__global__ void swiglu_fwd_kernel(const __nv_bfloat16* __restrict__ g,
                                  const __nv_bfloat16* __restrict__ u,
                                  __nv_bfloat16* __restrict__ act, int64_t n8) {
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < n8;
       e += (int64_t)gridDim.x * blockDim.x) {
    float a[8], b[8];
    load8(g + e * 8, a);
    load8(u + e * 8, b);
#pragma unroll
    for (int i = 0; i < 8; ++i) a[i] = swiglu_elem(a[i], b[i]);
    store8(act + e * 8, a);
  }
}

// dg = d * u * s * (1 + g (1 - s)),  du = d * g * s,   s = sigmoid(g)
__global__ void swiglu_bwd_kernel(const __nv_bfloat16* __restrict__ d,
                                  const __nv_bfloat16* __restrict__ g,
                                  const __nv_bfloat16* __restrict__ u,
                                  __nv_bfloat16* __restrict__ dg, __nv_bfloat16* __restrict__ du,
                                  int64_t n8) {
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < n8;
       e += (int64_t)gridDim.x * blockDim.x) {
    float dd[8], a[8], b[8], og[8], ou[8];
    load8(d + e * 8, dd);
    load8(g + e * 8, a);
    load8(u + e * 8, b);
#pragma unroll
    for (int i = 0; i < 8; ++i) swiglu_grad_elem(dd[i], a[i], b[i], og[i], ou[i]);
    store8(dg + e * 8, og);
    store8(du + e * 8, ou);
  }
}

int grid_1d(int64_t work, int num_sms) {
  int64_t b = (work + 255) / 256;
  const int64_t cap = static_cast<int64_t>(num_sms) * 16;
  return static_cast<int>(b < 1 ? 1 : (b > cap ? cap : b));
}

}  // namespace

int launch_rmsnorm_fwd(const void* x, const void* w, void* y, int64_t rows, int64_t cols,
                       float eps, cudaStream_t st) {
  const cudaError_t e = launch_pdl(rmsnorm_fwd_kernel, dim3(static_cast<unsigned>(rows)), dim3(kRowThreads), 0,
                                   st, static_cast<const __nv_bfloat16*>(x),
                                   static_cast<const __nv_bfloat16*>(w), static_cast<__nv_bfloat16*>(y),
                                   cols, eps);
  note_launch();
  return e == cudaSuccess ? FITQ_OK : FITQ_ERR_CUDA;
}

int launch_rmsnorm_bwd(const void* dy, const void* x, const void* w, void* dx, int64_t rows,
                       int64_t cols, float eps, cudaStream_t st) {
  rmsnorm_bwd_kernel<<<static_cast<unsigned>(rows), kRowThreads, 0, st>>>(
      static_cast<const __nv_bfloat16*>(dy), static_cast<const __nv_bfloat16*>(x),
      static_cast<const __nv_bfloat16*>(w), static_cast<__nv_bfloat16*>(dx), cols, eps);
  note_launch();
  return launch_result();
}

int launch_rope(const void* t, void* out, const float* cs, const float* sn, int64_t rows,
                int heads, int dim, int64_t seq, int backward, cudaStream_t st, int num_sms) {
  const int64_t work = rows * heads * (dim / 16);
  if (backward)
    rope_kernel<true><<<grid_1d(work, num_sms), 256, 0, st>>>(
        static_cast<const __nv_bfloat16*>(t), static_cast<__nv_bfloat16*>(out), cs, sn, rows,
        heads, dim, seq);
  else
    rope_kernel<false><<<grid_1d(work, num_sms), 256, 0, st>>>(
        static_cast<const __nv_bfloat16*>(t), static_cast<__nv_bfloat16*>(out), cs, sn, rows,
        heads, dim, seq);
  note_launch();
  return launch_result();
}

int launch_rope_append(const void* q, const void* k, const void* v, void* q_out, void* k_cache,
                       void* v_cache, const float* cs, const float* sn, int64_t batch, int t_new,
                       int heads, int kv_heads, int dim, int prefix, int cap, cudaStream_t st,
                       int num_sms) {
  const int64_t rows = batch * t_new;
  const int64_t work = rows * (heads + 2 * kv_heads) * (dim / 16);
  const cudaError_t e = launch_pdl(
      rope_append_kernel, dim3(grid_1d(work, num_sms)), dim3(256), 0, st, static_cast<const __nv_bfloat16*>(q),
      static_cast<const __nv_bfloat16*>(k), static_cast<const __nv_bfloat16*>(v),
      static_cast<__nv_bfloat16*>(q_out), static_cast<__nv_bfloat16*>(k_cache),
      static_cast<__nv_bfloat16*>(v_cache), cs, sn, rows, t_new, heads, kv_heads, dim, prefix, cap);
  note_launch();
  if (e != cudaSuccess) return FITQ_ERR_CUDA;
  return launch_result();
}

int launch_swiglu_fwd(const void* g, const void* u, void* act, int64_t n, cudaStream_t st,
                      int num_sms) {
  swiglu_fwd_kernel<<<grid_1d(n / 8, num_sms), 256, 0, st>>>(
      static_cast<const __nv_bfloat16*>(g), static_cast<const __nv_bfloat16*>(u),
      static_cast<__nv_bfloat16*>(act), n / 8);
  note_launch();
  return launch_result();
}

int launch_swiglu_bwd(const void* d, const void* g, const void* u, void* dg, void* du, int64_t n,
                      cudaStream_t st, int num_sms) {
  swiglu_bwd_kernel<<<grid_1d(n / 8, num_sms), 256, 0, st>>>(
      static_cast<const __nv_bfloat16*>(d), static_cast<const __nv_bfloat16*>(g),
      static_cast<const __nv_bfloat16*>(u), static_cast<__nv_bfloat16*>(dg),
      static_cast<__nv_bfloat16*>(du), n / 8);
  note_launch();
  return launch_result();
}

}  // namespace fitq
