// NF4 GEMV / skinny GEMM for decode and speculative-verify row counts
// (M <= 64): y[M,N] = x[M,K].W^T (+ LoRA) with W streamed once from HBM.
//
// Replaces bitsandbytes gemv_4bit (single-token path of matmul_4bit,
// fitllm/forward.py:623-625) and widens it to the verify shapes
// (fitllm/inference.py:380-397, M = batch x (draft+1)).
//
// The kernel is bound by how fast NF4 bytes can be turned into tensor-core
// operands, so the decode path is built around one cheap step per byte:
//   * the weights are the A operand of mma.sync m16n8k16 (16 weight rows per
//     warp tile), the activations x the B operand (n8 tiles of tokens);
//   * a packed byte holds two consecutive weights of one row, which is exactly
//     one bf16x2 A-fragment register: one `prmt` builds the shared-memory
//     address (byte << 8 | lane << 2) and one `ld.shared` returns the pair of
//     bf16 code values from a 256-entry table replicated per lane at a
//     256-byte stride (conflict-free), i.e. about one instruction per weight;
//   * a 64-column NF4 block shares one absmax, so the fp32 product of a block
//     (4 MMAs) is scaled once per row: w = code * absmax is applied to the
//     partial sum.  The GEMV output is held to the 1e-2 contract; the
//     bit-exact dequantised values are fitq_nf4_dequant's.
//
// Work decomposition: a CTA (16 warps) owns RT row tiles of 16 rows and one
// K slice of KC columns; its warps are RT row tiles x KW k-parts (RT*KW=16).
// Each thread streams 8 bytes of each of its two rows per block with 8-byte
// loads, double-buffered four blocks at a time; x for the slice is staged in
// shared memory once per CTA.  Warps of the same row tile are combined in a
// fixed order, and each slice writes fp32 partial sums that a finishing pass
// reduces in slice order (deterministic), adding LoRA, bias and residual.
#include "common.cuh"
#include "kernels.cuh"

namespace fitq {
namespace {

constexpr int kWarps = 16;
constexpr int kThreads = kWarps * 32;
constexpr int kTableBytes = 256 * 256;  // entry e at e*256, lane l at +4l
constexpr int kChunk = 4;               // blocks per double-buffer chunk

__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
      "{%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t lds32(uint32_t addr) {
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(addr));
  return v;
}

__device__ __forceinline__ uint4 lds128(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(addr));
  return v;
}

// Table offset of byte j of v: (byte << 8) | (lane << 2), built with one prmt
// from v and lane4 = lane << 2 (lane4 < 256 fits its low byte).
template <int J>
__device__ __forceinline__ uint32_t lut_off(uint32_t v, uint32_t lane4) {
  uint32_t r;
  // selector: out byte0 <- lane4 byte0 (index 4), out byte1 <- v byte J, bytes 2,3 <- lane4 byte 1 (0)
  constexpr uint32_t sel = 0x5500u | (static_cast<uint32_t>(J) << 4) | 4u;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(v), "r"(lane4), "n"(sel));
  return r;
}

__device__ __forceinline__ float block_absmax(const Nf4Args& w, int64_t blk, const float* s_nqm) {
  if (w.absmax_f32 != nullptr) return __ldg(w.absmax_f32 + blk);
  return __fadd_rn(__fmul_rn(s_nqm[__ldg(w.absmax_code + blk)], __ldg(w.nested_absmax + (blk >> 8))),
                   w.offset);
}

// Work item = (K slice, group of RT row tiles); the grid is persistent (one
// CTA per SM builds the code table once) and walks items slice-major, staging
// the slice's x in shared memory whenever the slice changes.  The plan makes
// every warp's block range a whole number of CH-block chunks.
// partial[slice][m][n] = sum over the slice of x[m,k] * W[n,k]
extern __shared__ __align__(16) uint8_t g_gemv_smem[];

// bf16x2 code pair of byte J of v: table entry (byte << 8) | (lane << 2).
template <int J>
__device__ __forceinline__ uint32_t lut(uint32_t v, uint32_t lane4) {
  return *reinterpret_cast<const uint32_t*>(g_gemv_smem + lut_off<J>(v, lane4));
}

template <int NT8, int CH>
__global__ void __launch_bounds__(kThreads, 1)
    nf4_gemv_kernel(Nf4Args w, const __nv_bfloat16* __restrict__ x, int M, int rt, int kcb,
                    int row_groups, int n_items, float* __restrict__ partial) {
  __shared__ float s_nqm[256];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, q = lane & 3;
  const int kw = kWarps / rt;
  const int K = static_cast<int>(w.k_in), N = static_cast<int>(w.n_out);
  const int nblk = K / 64;
  const int xpitch = kcb * 64 + 8;  // bf16 elements per staged x row
  const int tok_n = NT8 * 8;

  uint32_t* table = reinterpret_cast<uint32_t*>(g_gemv_smem);
  __nv_bfloat16* xs = reinterpret_cast<__nv_bfloat16*>(g_gemv_smem + kTableBytes);
  float* red = reinterpret_cast<float*>(g_gemv_smem + kTableBytes + static_cast<size_t>(tok_n) * xpitch * 2);

  // table entry e = {bf16(qm[e >> 4]), bf16(qm[e & 15])}, 64 copies per entry (256-B stride)
  for (int i = threadIdx.x; i < 256 * 64; i += kThreads) {
    const int e = i >> 6;
    table[i] = pack_bf16x2(w.quant_map[e >> 4], w.quant_map[e & 15]);
  }
  if (threadIdx.x < 256 && w.nested_quant_map != nullptr)
    s_nqm[threadIdx.x] = w.nested_quant_map[threadIdx.x];
  const bool nested = w.absmax_f32 == nullptr;

  const int tile = warp % rt, part = warp / rt;
  const uint32_t lane4 = static_cast<uint32_t>(lane) << 2;
  const uint32_t xbase = smem_u32(xs);
  int cur_slice = -1;

  for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
    const int slice = item / row_groups, rg = item % row_groups;
    const int kb0 = slice * kcb;
    const int nb = min(kcb, nblk - kb0);
    if (slice != cur_slice) {
      __syncthreads();  // previous slice's x no longer read
      const int vec_per_row = nb * 8;
      for (int i = threadIdx.x; i < tok_n * vec_per_row; i += kThreads) {
        const int r = i / vec_per_row, c = (i % vec_per_row) * 8;
        uint4 v = make_uint4(0, 0, 0, 0);
        if (r < M)
          v = __ldg(reinterpret_cast<const uint4*>(x + static_cast<int64_t>(r) * K + kb0 * 64 + c));
        *reinterpret_cast<uint4*>(xs + r * xpitch + c) = v;
      }
      __syncthreads();
      cur_slice = slice;
    }
    const int ra = rg * rt * 16 + tile * 16 + g, rb = ra + 8;
    const int per = nb / kw;  // a multiple of CH (plan)
    const int wb0 = part * per;
    // byte offsets (fit in 32 bits: N*K/2 < 2^31) of this thread's 8 bytes in block kb0+wb0
    const uint8_t* pa = w.packed + ((ra * nblk + kb0 + wb0) * 32 + 8 * q);
    const uint8_t* pb = w.packed + ((rb * nblk + kb0 + wb0) * 32 + 8 * q);
    const int ba0 = ra * nblk + kb0 + wb0, bb0 = rb * nblk + kb0 + wb0;  // flat block ids

    float acc[NT8][4];
#pragma unroll
    for (int t = 0; t < NT8; ++t)
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[t][i] = 0.f;

    struct Chunk {
      uint2 wa[CH], wb[CH];
      uint32_t ca, cb;
      float na0, na1, nb0, nb1;
    };
    Chunk bufA, bufB;
    auto load_chunk = [&](Chunk& ck, int c0) {  // c0: block index relative to wb0
#pragma unroll
      for (int c = 0; c < CH; ++c) {
        ck.wa[c] = __ldg(reinterpret_cast<const uint2*>(pa + (c0 + c) * 32));
        ck.wb[c] = __ldg(reinterpret_cast<const uint2*>(pb + (c0 + c) * 32));
      }
      if (nested) {
        if (CH == 4) {
          ck.ca = __ldg(reinterpret_cast<const uint32_t*>(w.absmax_code + ba0 + c0));
          ck.cb = __ldg(reinterpret_cast<const uint32_t*>(w.absmax_code + bb0 + c0));
        } else {
          ck.ca = __ldg(reinterpret_cast<const uint16_t*>(w.absmax_code + ba0 + c0));
          ck.cb = __ldg(reinterpret_cast<const uint16_t*>(w.absmax_code + bb0 + c0));
        }
        ck.na0 = __ldg(w.nested_absmax + ((ba0 + c0) >> 8));
        ck.na1 = __ldg(w.nested_absmax + ((ba0 + c0 + CH - 1) >> 8));
        ck.nb0 = __ldg(w.nested_absmax + ((bb0 + c0) >> 8));
        ck.nb1 = __ldg(w.nested_absmax + ((bb0 + c0 + CH - 1) >> 8));
      }
    };
    auto compute_chunk = [&](const Chunk& ck, int c0) {
#pragma unroll
      for (int c = 0; c < CH; ++c) {
        float am_a, am_b;
        if (nested) {
          const float nsa = ((ba0 + c0 + c) >> 8) == ((ba0 + c0) >> 8) ? ck.na0 : ck.na1;
          const float nsb = ((bb0 + c0 + c) >> 8) == ((bb0 + c0) >> 8) ? ck.nb0 : ck.nb1;
          am_a = __fadd_rn(__fmul_rn(s_nqm[(ck.ca >> (8 * c)) & 0xFFu], nsa), w.offset);
          am_b = __fadd_rn(__fmul_rn(s_nqm[(ck.cb >> (8 * c)) & 0xFFu], nsb), w.offset);
        } else {
          am_a = __ldg(w.absmax_f32 + ba0 + c0 + c);
          am_b = __ldg(w.absmax_f32 + bb0 + c0 + c);
        }
        const uint2 wa = ck.wa[c], wbv = ck.wb[c];
        const uint32_t xcol = static_cast<uint32_t>((wb0 + c0 + c) * 64 + 16 * q) * 2;
#pragma unroll
        for (int t = 0; t < NT8; ++t) {
          const uint32_t xa = xbase + static_cast<uint32_t>((8 * t + g) * xpitch) * 2 + xcol;
          const uint4 x0 = lds128(xa), x1 = lds128(xa + 16);
          float tmp[4] = {0.f, 0.f, 0.f, 0.f};
          // A: byte 2i -> rows (g, g+8) cols 16q+4i+{0,1}; byte 2i+1 -> cols 16q+4i+{2,3}
          mma16816(tmp, lut<0>(wa.x, lane4), lut<0>(wbv.x, lane4), lut<1>(wa.x, lane4),
                   lut<1>(wbv.x, lane4), x0.x, x0.y);
          mma16816(tmp, lut<2>(wa.x, lane4), lut<2>(wbv.x, lane4), lut<3>(wa.x, lane4),
                   lut<3>(wbv.x, lane4), x0.z, x0.w);
          mma16816(tmp, lut<0>(wa.y, lane4), lut<0>(wbv.y, lane4), lut<1>(wa.y, lane4),
                   lut<1>(wbv.y, lane4), x1.x, x1.y);
          mma16816(tmp, lut<2>(wa.y, lane4), lut<2>(wbv.y, lane4), lut<3>(wa.y, lane4),
                   lut<3>(wbv.y, lane4), x1.z, x1.w);
          acc[t][0] = fmaf(tmp[0], am_a, acc[t][0]);
          acc[t][1] = fmaf(tmp[1], am_a, acc[t][1]);
          acc[t][2] = fmaf(tmp[2], am_b, acc[t][2]);
          acc[t][3] = fmaf(tmp[3], am_b, acc[t][3]);
        }
      }
    };

    load_chunk(bufA, 0);
    for (int c0 = 0; c0 < per; c0 += 2 * CH) {
      if (c0 + CH < per) load_chunk(bufB, c0 + CH);
      compute_chunk(bufA, c0);
      if (c0 + 2 * CH < per) load_chunk(bufA, c0 + 2 * CH);
      if (c0 + CH < per) compute_chunk(bufB, c0 + CH);
    }

    float* out = partial + static_cast<int64_t>(slice) * M * N;
    if (kw == 1) {
#pragma unroll
      for (int t = 0; t < NT8; ++t)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int n = (i >= 2 ? rb : ra);
          const int tk = 8 * t + 2 * q + (i & 1);
          if (tk < M) out[static_cast<int64_t>(tk) * N + n] = acc[t][i];
        }
    } else {
      for (int p = 0; p < kw; ++p) {
        if (part == p) {
#pragma unroll
          for (int t = 0; t < NT8; ++t)
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const int rr = g + (i >= 2 ? 8 : 0);
              const int tk = 8 * t + 2 * q + (i & 1);
              float& r = red[(tile * 16 + rr) * tok_n + tk];
              r = (p == 0) ? acc[t][i] : r + acc[t][i];
            }
        }
        __syncthreads();
      }
      const int nrow0 = rg * rt * 16;
      for (int e = threadIdx.x; e < rt * 16 * tok_n; e += kThreads) {
        const int rr = e / tok_n, tk = e % tok_n;
        if (tk < M) out[static_cast<int64_t>(tk) * N + nrow0 + rr] = red[e];
      }
      __syncthreads();
    }
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

struct Plan {
  int nt8, rt, kcb, ch;
  int64_t slices, row_groups;
  size_t smem;
};

size_t plan_smem(int nt8, int rt, int kcb) {
  const size_t xbytes = static_cast<size_t>(nt8 * 8) * (kcb * 64 + 8) * 2;
  const size_t red = rt > 0 && rt < kWarps ? static_cast<size_t>(rt) * 16 * nt8 * 8 * 4 : 0;
  return kTableBytes + xbytes + red;
}

// Row tiles per work item (RT) and K-slice blocks (kcb): enough items for two
// per SM when possible, then the fewest slices (least partial-sum traffic).
Plan make_plan(int64_t m, int64_t N, int64_t K, int num_sms) {
  Plan best{0, 0, 0, 0, 0, 0, 0};
  const int nt8 = static_cast<int>((m + 7) / 8);
  const int ch = nt8 <= 2 ? 4 : 2;
  const int64_t nblk = K / 64;
  int64_t best_items = -1;
  size_t best_partial = 0;
  const int rts[3] = {16, 8, 4};
  const int kcbs[6] = {128, 64, 32, 16, 8, 4};
  for (int ri = 0; ri < 3; ++ri) {
    const int rt = rts[ri];
    const int kw = kWarps / rt;
    if (N % (16 * rt) != 0) continue;
    for (int ki = 0; ki < 6; ++ki) {
      int kcb = kcbs[ki];
      if (kcb % (kw * ch) != 0 || nblk % (kw * ch) != 0) continue;
      if (kcb > nblk) kcb = static_cast<int>(nblk);
      if (plan_smem(nt8, rt, kcb) > 200 * 1024) continue;
      const int64_t slices = (nblk + kcb - 1) / kcb;
      const int64_t items = (N / (16 * rt)) * slices;
      const size_t partial = static_cast<size_t>(slices) * m * N * 4;
      const bool enough = items >= 2 * num_sms, best_enough = best_items >= 2 * num_sms;
      bool take = false;
      if (best_items < 0) take = true;
      else if (enough && !best_enough) take = true;
      else if (enough && best_enough) take = partial < best_partial;
      else if (!enough && !best_enough) take = items > best_items;
      if (take) {
        best = Plan{nt8, rt, kcb, ch, slices, N / (16 * rt), plan_smem(nt8, rt, kcb)};
        best_items = items;
        best_partial = partial;
      }
    }
  }
  return best;
}

}  // namespace

size_t gemv_partial_bytes(int64_t m, int64_t n_out, int64_t k_in, int num_sms, int* splits_out) {
  const Plan p = make_plan(m, n_out, k_in, num_sms);
  if (splits_out) *splits_out = static_cast<int>(p.slices);
  return static_cast<size_t>(p.slices * m * n_out) * sizeof(float);
}

int launch_nf4_gemv_core(const Nf4Args& w, const void* x, int64_t m, float* partial,
                         cudaStream_t st, int num_sms, int* splits_out) {
  const Plan p = make_plan(m, w.n_out, w.k_in, num_sms);
  if (p.rt == 0 || p.nt8 < 1 || p.nt8 > 8) return FITQ_ERR_UNSUPPORTED;
  if ((w.k_in / 64) % 4 != 0 || w.n_out * w.k_in / 2 >= (1ll << 31)) return FITQ_ERR_UNSUPPORTED;
  const int64_t items = p.row_groups * p.slices;
  const int grid = static_cast<int>(items < num_sms ? items : num_sms);
  auto xb = static_cast<const __nv_bfloat16*>(x);
  const int M = static_cast<int>(m);
  static bool attr[9][2] = {};
  cudaError_t e = cudaSuccess;
#define FITQ_GEMV_CASE(T, C)                                                                      \
  if (p.nt8 == T && p.ch == C) {                                                                  \
    if (!attr[T][C / 4]) {                                                                        \
      e = cudaFuncSetAttribute(nf4_gemv_kernel<T, C>,                                             \
                               cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);          \
      attr[T][C / 4] = (e == cudaSuccess);                                                        \
    }                                                                                             \
    nf4_gemv_kernel<T, C><<<grid, kThreads, p.smem, st>>>(w, xb, M, p.rt, p.kcb,                  \
                                                           static_cast<int>(p.row_groups),        \
                                                           static_cast<int>(items), partial);     \
    note_launch();                                                                                \
  }
  FITQ_GEMV_CASE(1, 4)
  FITQ_GEMV_CASE(2, 4)
  FITQ_GEMV_CASE(3, 2)
  FITQ_GEMV_CASE(4, 2)
  FITQ_GEMV_CASE(5, 2)
  FITQ_GEMV_CASE(6, 2)
  FITQ_GEMV_CASE(7, 2)
  FITQ_GEMV_CASE(8, 2)
#undef FITQ_GEMV_CASE
  if (e != cudaSuccess) return FITQ_ERR_CUDA;
  *splits_out = static_cast<int>(p.slices);
  return cudaGetLastError() == cudaSuccess ? FITQ_OK : FITQ_ERR_CUDA;
}

int launch_gemv_finish(const float* partial, int splits, int64_t m, int64_t n, const void* t_pad,
                       const float* lora_b, int rank, float scale, const void* bias,
                       const void* y_add, void* y, cudaStream_t st, int num_sms) {
  const int64_t total = m * n;
  int64_t blocks = (total + 255) / 256;
  if (blocks > static_cast<int64_t>(num_sms) * 8) blocks = static_cast<int64_t>(num_sms) * 8;
  if (blocks < 1) blocks = 1;
  gemv_finish_kernel<<<static_cast<int>(blocks), 256, 0, st>>>(
      partial, splits, static_cast<int>(m), n, static_cast<const __nv_bfloat16*>(t_pad), lora_b,
      rank, scale, static_cast<const __nv_bfloat16*>(bias), static_cast<const __nv_bfloat16*>(y_add),
      static_cast<__nv_bfloat16*>(y));
  note_launch();
  return cudaGetLastError() == cudaSuccess ? FITQ_OK : FITQ_ERR_CUDA;
}

}  // namespace fitq
