// NF4 GEMV / skinny GEMM for decode and speculative-verify row counts
// (M <= 64): y[M,N] = x[M,K].W^T (+ LoRA) with W streamed once from HBM.
//
// Replaces bitsandbytes gemv_4bit (single-token path of matmul_4bit,
// fitllm/forward.py:623-625) and widens it to the verify shapes
// (fitllm/inference.py:380-397, M = batch x (draft+1)).
//
// Layout of the work: a CTA owns 64 weight rows and one K range; its 8 warps
// take interleaved 64-column NF4 blocks of that range.  Per block a thread
// reads 8 packed bytes (16 weights) of one row for each of the 8 n8-tiles.
// The tensor-core product uses x as the A operand (m16 tiles) and the raw NF4
// codes as the B operand: byte -> two bf16 code values through a 256-entry
// table replicated per lane in shared memory (conflict-free, 1.5 instructions
// per weight).  Because a 64-column block shares one absmax, the fp32 block
// product is scaled by absmax once per block (the GEMV output is held to the
// 1e-2 contract; the bit-exact dequantised values are fitq_nf4_dequant's).
#include "common.cuh"
#include "kernels.cuh"

namespace fitq {
namespace {

constexpr int kGemvWarps = 8;
constexpr int kRowsPerCta = 64;  // largest row tile (MT <= 2); MT >= 3 uses 32 rows
__host__ __device__ constexpr int gemv_tiles(int mt) { return mt <= 2 ? 8 : 4; }

__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
      "{%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t lds32(uint32_t addr) {
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(addr));
  return v;
}

// partial[split][m][n] = sum over this CTA's K range of x[m,k] * W[n,k]
template <int MT>
__global__ void __launch_bounds__(kGemvWarps * 32) nf4_gemv_kernel(Nf4Args w,
                                                                   const __nv_bfloat16* __restrict__ x,
                                                                   int M, int kb_per_split,
                                                                   float* __restrict__ partial) {
  extern __shared__ __align__(16) uint8_t gsm[];
  // [0, 32 KB): table[e][lane] (e = packed byte) ; then reduction buffer
  uint32_t* table = reinterpret_cast<uint32_t*>(gsm);
  float* red = reinterpret_cast<float*>(gsm + 32768);  // [64 rows][MT*16 cols]
  __shared__ float s_nqm[256];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, q = lane & 3;
  {
    // entry e: low half = bf16(qm[e >> 4]) (element 2i), high half = bf16(qm[e & 15])
    const int e = threadIdx.x;  // 256 threads, one entry each
    const float lo = w.quant_map[e >> 4], hi = w.quant_map[e & 15];
    const uint32_t v = pack_bf16x2(lo, hi);
#pragma unroll 4
    for (int l = 0; l < 32; ++l) table[e * 32 + l] = v;
    if (w.nested_quant_map != nullptr) s_nqm[threadIdx.x] = w.nested_quant_map[threadIdx.x];
  }
  __syncthreads();
  const uint32_t tbase = smem_u32(table);
  const uint32_t l4 = static_cast<uint32_t>(lane) * 4u;  // entry e of lane l at e*128 + l*4

  const int64_t K = w.k_in, N = w.n_out;
  constexpr int NT = gemv_tiles(MT);
  const int64_t n0 = static_cast<int64_t>(blockIdx.x) * (8 * NT);
  const int64_t nblk = K / 64;
  const int64_t kb_begin = static_cast<int64_t>(blockIdx.y) * kb_per_split;
  const int64_t kb_end = kb_begin + kb_per_split < nblk ? kb_begin + kb_per_split : nblk;

  float acc[NT][MT][4];
#pragma unroll
  for (int t = 0; t < NT; ++t)
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[t][mt][i] = 0.f;

  for (int64_t kb = kb_begin + warp; kb < kb_end; kb += kGemvWarps) {
    // A fragments (x): MMA i of the block uses, for thread (g, q), columns
    // 16q + 4i + {0,1} (a0/a1) and 16q + 4i + {2,3} (a2/a3); the NF4 codes in
    // the B fragments are permuted the same way.
    uint32_t af[MT][4][4];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
      const int r0 = mt * 16 + g, r1 = r0 + 8;
      uint4 v0a = make_uint4(0, 0, 0, 0), v0b = v0a, v1a = v0a, v1b = v0a;
      const int64_t col = kb * 64 + 16 * q;
      if (r0 < M) {
        v0a = __ldg(reinterpret_cast<const uint4*>(x + r0 * K + col));
        v0b = __ldg(reinterpret_cast<const uint4*>(x + r0 * K + col + 8));
      }
      if (r1 < M) {
        v1a = __ldg(reinterpret_cast<const uint4*>(x + r1 * K + col));
        v1b = __ldg(reinterpret_cast<const uint4*>(x + r1 * K + col + 8));
      }
      const uint32_t r0w[8] = {v0a.x, v0a.y, v0a.z, v0a.w, v0b.x, v0b.y, v0b.z, v0b.w};
      const uint32_t r1w[8] = {v1a.x, v1a.y, v1a.z, v1a.w, v1b.x, v1b.y, v1b.z, v1b.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        af[mt][i][0] = r0w[2 * i];
        af[mt][i][1] = r1w[2 * i];
        af[mt][i][2] = r0w[2 * i + 1];
        af[mt][i][3] = r1w[2 * i + 1];
      }
    }
    // absmax of row (n0 + 8t + g) for this block; the scaling needs rows 2q, 2q+1.
#pragma unroll
    for (int t = 0; t < NT; ++t) {
      const int64_t row = n0 + 8 * t + g;
      const int64_t blk = row * nblk + kb;
      float am;
      if (w.absmax_f32 != nullptr) {
        am = __ldg(w.absmax_f32 + blk);
      } else {
        am = __fadd_rn(__fmul_rn(s_nqm[__ldg(w.absmax_code + blk)], __ldg(w.nested_absmax + (blk >> 8))),
                       w.offset);
      }
      const uint2 pk = __ldg(reinterpret_cast<const uint2*>(w.packed + (blk * 64 + 16 * q) / 2));
      const uint32_t qw[2] = {pk.x, pk.y};
      uint32_t bf[8];  // bf16x2 code pairs, columns 16q + 2j, +1
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const uint32_t v = qw[h];
        bf[4 * h + 0] = lds32(tbase + (((v << 7) & 0x7F80u) | l4));
        bf[4 * h + 1] = lds32(tbase + (((v >> 1) & 0x7F80u) | l4));
        bf[4 * h + 2] = lds32(tbase + (((v >> 9) & 0x7F80u) | l4));
        bf[4 * h + 3] = lds32(tbase + (((v >> 17) & 0x7F80u) | l4));
      }
      const float am_a = __shfl_sync(0xffffffffu, am, (2 * q) * 4);
      const float am_b = __shfl_sync(0xffffffffu, am, (2 * q + 1) * 4);
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        float tmp[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int i = 0; i < 4; ++i) mma16816(tmp, af[mt][i], bf[2 * i], bf[2 * i + 1]);
        acc[t][mt][0] = fmaf(tmp[0], am_a, acc[t][mt][0]);
        acc[t][mt][1] = fmaf(tmp[1], am_b, acc[t][mt][1]);
        acc[t][mt][2] = fmaf(tmp[2], am_a, acc[t][mt][2]);
        acc[t][mt][3] = fmaf(tmp[3], am_b, acc[t][mt][3]);
      }
    }
  }
  // Fixed-order reduction of the 8 warps: red[row (0..63)][m (0..MT*16)]
  constexpr int RC = MT * 16;
  for (int wv = 0; wv < kGemvWarps; ++wv) {
    if (warp == wv) {
#pragma unroll
      for (int t = 0; t < NT; ++t)
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int m = mt * 16 + g + (i >= 2 ? 8 : 0);
            const int nn = 8 * t + 2 * q + (i & 1);
            float& r = red[nn * RC + m];
            r = (wv == 0) ? acc[t][mt][i] : r + acc[t][mt][i];
          }
    }
    __syncthreads();
  }
  for (int e = threadIdx.x; e < 8 * NT * RC; e += kGemvWarps * 32) {
    const int nn = e / RC, m = e % RC;
    const int64_t n = n0 + nn;
    if (m < M && n < N) partial[(static_cast<int64_t>(blockIdx.y) * M + m) * N + n] = red[e];
  }
}

// y[m,n] = bf16( sum_s partial[s][m][n] + scale * sum_j T[m][j] * B[n][j] + bias[n] + y_add[m][n] )
__global__ void gemv_finish_kernel(const float* __restrict__ partial, int splits, int M,
                                   int64_t N, const __nv_bfloat16* __restrict__ t_pad,
                                   const float* __restrict__ lora_b, int rank, float scale,
                                   const __nv_bfloat16* __restrict__ bias,
                                   const __nv_bfloat16* __restrict__ y_add,
                                   __nv_bfloat16* __restrict__ y) {
  const int64_t total = static_cast<int64_t>(M) * N;
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total;
       e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t m = e / N, n = e % N;
    float s = 0.f;
    for (int sp = 0; sp < splits; ++sp) s += partial[sp * total + e];
    if (rank > 0) {
      float l = 0.f;
      for (int j = 0; j < rank; ++j)
        l = fmaf(__bfloat162float(t_pad[m * 64 + j]), lora_b[n * rank + j], l);
      s += scale * l;
    }
    if (bias) s += __bfloat162float(bias[n]);
    if (y_add) s += __bfloat162float(y_add[e]);
    y[e] = __float2bfloat16_rn(s);
  }
}

}  // namespace

size_t gemv_partial_bytes(int64_t m, int64_t n_out, int64_t k_in, int num_sms, int* splits_out) {
  const int64_t rows = 8 * gemv_tiles(static_cast<int>((m + 15) / 16));
  const int64_t row_groups = (n_out + rows - 1) / rows;
  const int64_t nblk = k_in / 64;
  int64_t splits = (2 * static_cast<int64_t>(num_sms) + row_groups - 1) / row_groups;
  const int64_t max_splits = (nblk + kGemvWarps - 1) / kGemvWarps;  // >= 8 blocks per split
  if (splits > max_splits) splits = max_splits;
  if (splits < 1) splits = 1;
  int64_t per = (nblk + splits - 1) / splits;
  splits = (nblk + per - 1) / per;
  if (splits_out) *splits_out = static_cast<int>(splits);
  return static_cast<size_t>(splits * m * n_out) * sizeof(float);
}

int launch_nf4_gemv_core(const Nf4Args& w, const void* x, int64_t m, float* partial,
                         cudaStream_t st, int num_sms, int* splits_out) {
  int splits = 1;
  gemv_partial_bytes(m, w.n_out, w.k_in, num_sms, &splits);
  const int64_t nblk = w.k_in / 64;
  const int per = static_cast<int>((nblk + splits - 1) / splits);
  const int mt = static_cast<int>((m + 15) / 16);
  const int64_t rows = 8 * gemv_tiles(mt);
  dim3 grid(static_cast<unsigned>((w.n_out + rows - 1) / rows), static_cast<unsigned>(splits));
  const size_t smem = 32768 + static_cast<size_t>(rows) * mt * 16 * sizeof(float);
  auto xb = static_cast<const __nv_bfloat16*>(x);
  const int M = static_cast<int>(m);
  static bool attr[5] = {false, false, false, false, false};
  cudaError_t e = cudaSuccess;
#define FITQ_GEMV_CASE(T)                                                                        \
  case T:                                                                                        \
    if (!attr[T]) {                                                                              \
      e = cudaFuncSetAttribute(nf4_gemv_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, \
                               static_cast<int>(32768 + kRowsPerCta * 4 * 16 * sizeof(float))); \
      attr[T] = (e == cudaSuccess);                                                              \
    }                                                                                            \
    nf4_gemv_kernel<T><<<grid, kGemvWarps * 32, smem, st>>>(w, xb, M, per, partial);             \
    note_launch();                                                                               \
    break;
  switch (mt) {
    FITQ_GEMV_CASE(1)
    FITQ_GEMV_CASE(2)
    FITQ_GEMV_CASE(3)
    FITQ_GEMV_CASE(4)
    default: return FITQ_ERR_UNSUPPORTED;
  }
#undef FITQ_GEMV_CASE
  if (e != cudaSuccess) return FITQ_ERR_CUDA;
  *splits_out = splits;
  return cudaGetLastError() == cudaSuccess ? FITQ_OK : FITQ_ERR_CUDA;
}

int launch_gemv_finish(const float* partial, int splits, int64_t m, int64_t n, const void* t_pad,
                       const float* lora_b, int rank, float scale, const void* bias,
                       const void* y_add, void* y,
                       cudaStream_t st, int num_sms) {
  const int64_t total = m * n;
  int64_t blocks = (total + 255) / 256;
  if (blocks > static_cast<int64_t>(num_sms) * 8) blocks = static_cast<int64_t>(num_sms) * 8;
  gemv_finish_kernel<<<static_cast<int>(blocks), 256, 0, st>>>(
      partial, splits, static_cast<int>(m), n, static_cast<const __nv_bfloat16*>(t_pad), lora_b,
      rank, scale, static_cast<const __nv_bfloat16*>(bias), static_cast<const __nv_bfloat16*>(y_add),
      static_cast<__nv_bfloat16*>(y));
  note_launch();
  return cudaGetLastError() == cudaSuccess ? FITQ_OK : FITQ_ERR_CUDA;
}

}  // namespace fitq
