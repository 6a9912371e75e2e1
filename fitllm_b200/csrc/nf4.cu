// NF4 dequantisation (bit-exact) and quantisation kernels.
//
// Dequant follows bitsandbytes' dequantize_4bit with a double-quantised
// QuantState, as FitLLM restores it from shard keys (fitllm/forward.py:76-109):
// absmax_b = fl(fl(nested_quant_map[code_b] * nested_absmax[b / 256]) + offset)
// (blockwise dequant then "+= offset": two roundings, no FMA), then
// w = fl(quant_map[nibble] * absmax_b) rounded to nearest even into bf16/fp16.
// The quantiser is this project's restatement of blockwise NF4 (block 64)
// plus 8-bit dynamic double quantisation (block 256); its decision rule and
// offset summation order are fixed so that host and device agree bit for bit.
#include "common.cuh"
#include "kernels.cuh"

namespace fitq {

// Decoded fp32 absmax of NF4 block b (either storage form).
__device__ __forceinline__ float absmax_of_block(const Nf4Args& w, int64_t b,
                                                 const float* s_nqm) {
  if (w.absmax_f32 != nullptr) return __ldg(w.absmax_f32 + b);
  float p = __fmul_rn(s_nqm[__ldg(w.absmax_code + b)], __ldg(w.nested_absmax + (b >> 8)));
  return __fadd_rn(p, w.offset);
}

template <typename OutT>
__device__ __forceinline__ uint32_t pack2(float lo, float hi);
template <>
__device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float lo, float hi) {
  return pack_bf16x2(lo, hi);
}
template <>
__device__ __forceinline__ uint32_t pack2<__half>(float lo, float hi) {
  __half2 v = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// Each thread: 32 consecutive weights = 16 packed bytes -> 64 output bytes.
template <typename OutT>
__global__ void __launch_bounds__(256) nf4_dequant_kernel(Nf4Args w, OutT* __restrict__ out,
                                                          int64_t n_items) {
  __shared__ float s_qm[16];
  __shared__ float s_nqm[256];
  pdl_launch_dependents();
  pdl_wait();  // out may still be read by the previous kernel
  if (threadIdx.x < 16) s_qm[threadIdx.x] = w.quant_map[threadIdx.x];
  if (w.nested_quant_map != nullptr) s_nqm[threadIdx.x] = w.nested_quant_map[threadIdx.x];
  __syncthreads();
  // Four items per thread per pass, their loads issued together: one item's
  // load-to-use latency alone left HBM half idle.
  constexpr int U = 4;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t it0 = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; it0 < n_items; it0 += U * stride) {
    uint4 q[U];
    float am[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t it = it0 + u * stride;
      if (it < n_items) q[u] = __ldg(reinterpret_cast<const uint4*>(w.packed) + it);
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t it = it0 + u * stride;
      am[u] = it < n_items ? absmax_of_block(w, it >> 1, s_nqm) : 0.f;
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t it = it0 + u * stride;
      if (it >= n_items) break;
      const uint32_t words[4] = {q[u].x, q[u].y, q[u].z, q[u].w};
      uint32_t o[16];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
#pragma unroll
        for (int b = 0; b < 4; ++b) {
          uint32_t byte = (words[j] >> (8 * b)) & 0xFFu;
          float hi = __fmul_rn(s_qm[byte >> 4], am[u]);
          float lo = __fmul_rn(s_qm[byte & 0xF], am[u]);
          o[j * 4 + b] = pack2<OutT>(hi, lo);  // element 2i (high nibble) first in memory
        }
      }
      uint4* dst = reinterpret_cast<uint4*>(out) + it * 4;
#pragma unroll
      for (int v = 0; v < 4; ++v) dst[v] = make_uint4(o[4 * v], o[4 * v + 1], o[4 * v + 2], o[4 * v + 3]);
    }
  }
}

// Transposed dequant: out[K,N] = W^T.  Tile = 64 rows of W (n) x 64 columns
// (k, exactly one NF4 block per row); 256 threads, each 16 weights of one row.
template <typename OutT>
__global__ void __launch_bounds__(256) nf4_dequant_t_kernel(Nf4Args w, OutT* __restrict__ out) {
  __shared__ float s_qm[16];
  __shared__ float s_nqm[256];
  pdl_launch_dependents();
  pdl_wait();  // out may still be read by the previous kernel
  // [tile of the pass][k][n], padded rows; two tiles per pass, their loads
  // issued together (one 8-byte load in flight per thread left HBM idle)
  __shared__ uint16_t s_t[2][64][64 + 8];
  if (threadIdx.x < 16) s_qm[threadIdx.x] = w.quant_map[threadIdx.x];
  if (w.nested_quant_map != nullptr) s_nqm[threadIdx.x] = w.nested_quant_map[threadIdx.x];
  __syncthreads();
  const int64_t N = w.n_out, K = w.k_in;
  const int64_t tiles_k = K / 64;
  const int64_t n_tiles = (N / 64) * tiles_k;
  const int r = threadIdx.x >> 2;  // row n0 + r
  const int part = threadIdx.x & 3;  // weights k0 + 16*part .. +15
  for (int64_t tile0 = blockIdx.x; tile0 < n_tiles; tile0 += 2 * (int64_t)gridDim.x) {
    uint2 q[2];
    float am[2];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int64_t tile = tile0 + u * (int64_t)gridDim.x;
      if (tile < n_tiles) {
        const int64_t n0 = (tile / tiles_k) * 64, k0 = (tile % tiles_k) * 64;
        const int64_t elem = (n0 + r) * K + k0 + 16 * part;
        q[u] = __ldg(reinterpret_cast<const uint2*>(w.packed + (elem >> 1)));
        am[u] = absmax_of_block(w, elem >> 6, s_nqm);
      }
    }
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      if (tile0 + u * (int64_t)gridDim.x >= n_tiles) break;  // block-uniform
      const uint32_t words[2] = {q[u].x, q[u].y};
#pragma unroll
      for (int j = 0; j < 2; ++j) {
#pragma unroll
        for (int b = 0; b < 4; ++b) {
          uint32_t byte = (words[j] >> (8 * b)) & 0xFFu;
          uint32_t p = pack2<OutT>(__fmul_rn(s_qm[byte >> 4], am[u]), __fmul_rn(s_qm[byte & 0xF], am[u]));
          // column rotated by 16*part: spreads the four parts over distinct banks
          int kk = 16 * part + 8 * j + 2 * b;
          int col = (r + 16 * part) & 63;
          s_t[u][kk][col] = static_cast<uint16_t>(p & 0xFFFFu);
          s_t[u][kk + 1][col] = static_cast<uint16_t>(p >> 16);
        }
      }
    }
    __syncthreads();
    // per tile: 64 rows (k) x 128 bytes: 8 threads per row, 16 bytes each.
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int64_t tile = tile0 + u * (int64_t)gridDim.x;
      if (tile >= n_tiles) break;  // block-uniform
      const int64_t n0 = (tile / tiles_k) * 64, k0 = (tile % tiles_k) * 64;
#pragma unroll
      for (int pass = 0; pass < 2; ++pass) {
        const int kr = (threadIdx.x >> 3) + 32 * pass;
        const int c8 = threadIdx.x & 7;
        const uint4 v = *reinterpret_cast<const uint4*>(&s_t[u][kr][(c8 * 8 + 16 * (kr >> 4)) & 63]);
        *reinterpret_cast<uint4*>(out + (k0 + kr) * N + n0 + c8 * 8) = v;
      }
    }
    __syncthreads();
  }
}

// ------------------------------------------------------------ quantisation
__device__ __forceinline__ int count_below(const float* t, int nt, float x) {
  int lo = 0, hi = nt;
  while (lo < hi) {
    int mid = (lo + hi) >> 1;
    if (t[mid] < x) lo = mid + 1; else hi = mid;
  }
  return lo;
}

// One warp per 64-element block: lane l holds elements 2l and 2l+1.
__global__ void __launch_bounds__(256) nf4_quant_blocks_kernel(const float* __restrict__ wt,
                                                               int64_t nb,
                                                               const float* __restrict__ qmap,
                                                               uint8_t* __restrict__ packed,
                                                               float* __restrict__ absmax) {
  __shared__ float s_t[15];
  if (threadIdx.x < 15)
    s_t[threadIdx.x] = __fmul_rn(0.5f, __fadd_rn(qmap[threadIdx.x], qmap[threadIdx.x + 1]));
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t b = blockIdx.x * (int64_t)(blockDim.x >> 5) + (threadIdx.x >> 5); b < nb; b += warps) {
    const float2 v = __ldg(reinterpret_cast<const float2*>(wt + b * 64) + lane);
    float am = fmaxf(fabsf(v.x), fabsf(v.y));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, o));
    const float inv = am > 0.0f ? __fdiv_rn(1.0f, am) : 0.0f;
    const int c0 = count_below(s_t, 15, __fmul_rn(v.x, inv));
    const int c1 = count_below(s_t, 15, __fmul_rn(v.y, inv));
    packed[b * 32 + lane] = static_cast<uint8_t>((c0 << 4) | c1);
    if (lane == 0) absmax[b] = am;
  }
}

// Partial sums of absmax in double over consecutive chunks of 4096, each
// accumulated strictly left to right (one thread per chunk).
__global__ void absmax_chunk_sum_kernel(const float* __restrict__ absmax, int64_t nb,
                                        double* __restrict__ partial) {
  const int64_t c = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  const int64_t s = c * kOffsetChunk;
  if (s >= nb) return;
  const int64_t e = s + kOffsetChunk < nb ? s + kOffsetChunk : nb;
  double acc = 0.0;
  for (int64_t i = s; i < e; ++i) acc = __dadd_rn(acc, (double)absmax[i]);
  partial[c] = acc;
}

__global__ void absmax_offset_kernel(const double* __restrict__ partial, int64_t nchunks,
                                     int64_t nb, float* __restrict__ offset_out) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  double t = 0.0;
  for (int64_t i = 0; i < nchunks; ++i) t = __dadd_rn(t, partial[i]);
  offset_out[0] = __double2float_rn(__ddiv_rn(t, (double)nb));
}

// One CTA (256 threads) per nested block of 256 absmax values.
__global__ void __launch_bounds__(256) dq_quant_kernel(const float* __restrict__ absmax, int64_t nb,
                                                       const float* __restrict__ nqmap,
                                                       const float* __restrict__ offset_ptr,
                                                       uint8_t* __restrict__ codes,
                                                       float* __restrict__ nested_absmax) {
  __shared__ float s_t[255];
  __shared__ float s_red[8];
  if (threadIdx.x < 255)
    s_t[threadIdx.x] = __fmul_rn(0.5f, __fadd_rn(nqmap[threadIdx.x], nqmap[threadIdx.x + 1]));
  const float offset = offset_ptr[0];
  const int64_t i = blockIdx.x * 256ll + threadIdx.x;
  const float c = i < nb ? __fsub_rn(absmax[i], offset) : 0.0f;
  float m = fabsf(c);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((threadIdx.x & 31) == 0) s_red[threadIdx.x >> 5] = m;
  __syncthreads();
  m = s_red[0];
#pragma unroll
  for (int k = 1; k < 8; ++k) m = fmaxf(m, s_red[k]);
  const float inv = m > 0.0f ? __fdiv_rn(1.0f, m) : 0.0f;
  if (i < nb) codes[i] = static_cast<uint8_t>(count_below(s_t, 255, __fmul_rn(c, inv)));
  if (threadIdx.x == 0) nested_absmax[blockIdx.x] = m;
}

// ------------------------------------------------------------ launchers
int launch_nf4_dequant(const Nf4Args& w, void* out, int out_dtype, int transpose,
                       cudaStream_t st, int num_sms) {
  const int64_t n = w.n_out * w.k_in;
  if (!transpose) {
    const int64_t items = n / 32;
    const int64_t want = (items + 255) / 256;
    const int grid = (int)(want < (int64_t)num_sms * 8 ? want : (int64_t)num_sms * 8);
    if (out_dtype == FITQ_DTYPE_BF16)
      launch_pdl(nf4_dequant_kernel<__nv_bfloat16>, dim3(grid), dim3(256), 0, st, w, (__nv_bfloat16*)out, items);
    else
      launch_pdl(nf4_dequant_kernel<__half>, dim3(grid), dim3(256), 0, st, w, (__half*)out, items);
    note_launch();
  } else {
    const int64_t tiles = (w.n_out / 64) * (w.k_in / 64);
    const int grid = (int)(tiles < (int64_t)num_sms * 8 ? tiles : (int64_t)num_sms * 8);
    if (out_dtype == FITQ_DTYPE_BF16)
      launch_pdl(nf4_dequant_t_kernel<__nv_bfloat16>, dim3(grid), dim3(256), 0, st, w, (__nv_bfloat16*)out);
    else
      launch_pdl(nf4_dequant_t_kernel<__half>, dim3(grid), dim3(256), 0, st, w, (__half*)out);
    note_launch();
  }
  return launch_result();
}

int launch_nf4_quantize(const float* wt, int64_t n, const float* qmap, const float* nqmap,
                        uint8_t* packed, uint8_t* codes, float* nested_absmax, float* offset_out,
                        float* absmax_ws, double* partial_ws, cudaStream_t st, int num_sms) {
  const int64_t nb = n / 64;
  {
    const int64_t want = (nb + 7) / 8;
    const int grid = (int)(want < (int64_t)num_sms * 16 ? want : (int64_t)num_sms * 16);
    nf4_quant_blocks_kernel<<<grid, 256, 0, st>>>(wt, nb, qmap, packed, absmax_ws);
    note_launch();
  }
  const int64_t nchunks = (nb + kOffsetChunk - 1) / kOffsetChunk;
  absmax_chunk_sum_kernel<<<(int)((nchunks + 127) / 128), 128, 0, st>>>(absmax_ws, nb, partial_ws);
  note_launch();
  absmax_offset_kernel<<<1, 32, 0, st>>>(partial_ws, nchunks, nb, offset_out);
  note_launch();
  const int64_t nn = (nb + 255) / 256;
  dq_quant_kernel<<<(int)nn, 256, 0, st>>>(absmax_ws, nb, nqmap, offset_out, codes, nested_absmax);
  note_launch();
  return launch_result();
}

}  // namespace fitq
