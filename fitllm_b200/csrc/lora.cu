// LoRA adapter kernels for the QLoRA linear (PEFT lora.Linear4bit semantics,
// fitllm/qlora.py:74-83): the rank-r projections T = x.A^T and U = dy.B, the
// row reductions dA = s.U^T.x and dB = s.dy^T.T, and the small casts that turn
// the fp32 adapter parameters into the bf16 operands of the tcgen05 GEMM.
#include "common.cuh"
#include "kernels.cuh"

namespace fitq {
namespace {

__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], uint32_t a0, uint32_t a1,
                                               uint32_t a2, uint32_t a3, uint32_t b0,
                                               uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
      "{%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// out[M, R] = in[M, D] . wt[R, D]^T with warp-level bf16 MMA (m16n8k16).
// A CTA owns 16 rows; its 4 warps take interleaved 32-column chunks of D and
// are reduced through shared memory in a fixed order.  Inside a chunk every
// thread loads 16 contiguous bytes of a row and feeds them to two MMAs: the
// reduction index is permuted identically in both operands, which leaves the
// sum unchanged and keeps every load coalesced.
template <int R>
__global__ void __launch_bounds__(128) lora_rowproj_kernel(const __nv_bfloat16* __restrict__ in,
                                                           int64_t ld, int64_t M, int64_t D,
                                                           const __nv_bfloat16* __restrict__ wt,
                                                           __nv_bfloat16* __restrict__ out_pad,
                                                           __nv_bfloat16* __restrict__ out_dense) {
  pdl_launch_dependents();
  pdl_wait();  // inputs are the previous kernels' outputs
  constexpr int NT = R / 8;
  __shared__ float red[4][16][R];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, q = lane & 3;
  const int64_t m0 = static_cast<int64_t>(blockIdx.x) * 16;
  const int64_t ra = m0 + g, rb = m0 + g + 8;
  float acc[NT][4];
#pragma unroll
  for (int t = 0; t < NT; ++t)
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[t][i] = 0.f;
  const int64_t nchunks = D / 32;
  const uint4 zero = make_uint4(0, 0, 0, 0);
  for (int64_t c = warp; c < nchunks; c += 4) {
    const int64_t col = c * 32 + 8 * q;
    const uint4 xa = ra < M ? __ldg(reinterpret_cast<const uint4*>(in + ra * ld + col)) : zero;
    const uint4 xb = rb < M ? __ldg(reinterpret_cast<const uint4*>(in + rb * ld + col)) : zero;
#pragma unroll
    for (int t = 0; t < NT; ++t) {
      const uint4 wb = __ldg(reinterpret_cast<const uint4*>(wt + (int64_t)(8 * t + g) * D + col));
      mma_bf16_16816(acc[t], xa.x, xb.x, xa.y, xb.y, wb.x, wb.y);
      mma_bf16_16816(acc[t], xa.z, xb.z, xa.w, xb.w, wb.z, wb.w);
    }
  }
#pragma unroll
  for (int t = 0; t < NT; ++t) {
    red[warp][g][8 * t + 2 * q] = acc[t][0];
    red[warp][g][8 * t + 2 * q + 1] = acc[t][1];
    red[warp][g + 8][8 * t + 2 * q] = acc[t][2];
    red[warp][g + 8][8 * t + 2 * q + 1] = acc[t][3];
  }
  __syncthreads();
  for (int e = threadIdx.x; e < 16 * R / 2; e += 128) {
    const int row = (2 * e) / R, col = (2 * e) % R;
    const int64_t m = m0 + row;
    if (m >= M) continue;
    float v0 = red[0][row][col], v1 = red[0][row][col + 1];
#pragma unroll
    for (int w = 1; w < 4; ++w) {
      v0 += red[w][row][col];
      v1 += red[w][row][col + 1];
    }
    const uint32_t pk = pack_bf16x2(v0, v1);
    *reinterpret_cast<uint32_t*>(out_pad + m * 64 + col) = pk;
    if (out_dense) *reinterpret_cast<uint32_t*>(out_dense + m * R + col) = pk;
  }
}

// Few-row variant of the projection (decode / verify, M <= 64): the D axis is
// split over gridDim.y slices of kRowprojSlice columns so that a handful of
// rows still spreads over many CTAs; partial[slice][m][j] in fp32, reduced by
// lora_rowproj_finish_kernel in slice order.
constexpr int kRowprojSlice = 512;

template <int R>
__global__ void __launch_bounds__(128) lora_rowproj_split_kernel(
    const __nv_bfloat16* __restrict__ in, int64_t ld, int64_t M, int64_t D,
    const __nv_bfloat16* __restrict__ wt, float* __restrict__ partial) {
  pdl_launch_dependents();
  pdl_wait();  // inputs are the previous kernels' outputs
  constexpr int NT = R / 8;
  __shared__ float red[4][16][R];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, q = lane & 3;
  const int64_t m0 = static_cast<int64_t>(blockIdx.x) * 16;
  const int64_t ra = m0 + g, rb = m0 + g + 8;
  const int64_t d0 = static_cast<int64_t>(blockIdx.y) * kRowprojSlice;
  const int64_t d1 = d0 + kRowprojSlice < D ? d0 + kRowprojSlice : D;
  float acc[NT][4];
#pragma unroll
  for (int t = 0; t < NT; ++t)
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[t][i] = 0.f;
  const uint4 zero = make_uint4(0, 0, 0, 0);
  for (int64_t col0 = d0 + warp * 32; col0 < d1; col0 += 128) {
    const int64_t col = col0 + 8 * q;
    const uint4 xa = ra < M ? __ldg(reinterpret_cast<const uint4*>(in + ra * ld + col)) : zero;
    const uint4 xb = rb < M ? __ldg(reinterpret_cast<const uint4*>(in + rb * ld + col)) : zero;
#pragma unroll
    for (int t = 0; t < NT; ++t) {
      const uint4 wb = __ldg(reinterpret_cast<const uint4*>(wt + (int64_t)(8 * t + g) * D + col));
      mma_bf16_16816(acc[t], xa.x, xb.x, xa.y, xb.y, wb.x, wb.y);
      mma_bf16_16816(acc[t], xa.z, xb.z, xa.w, xb.w, wb.z, wb.w);
    }
  }
#pragma unroll
  for (int t = 0; t < NT; ++t) {
    red[warp][g][8 * t + 2 * q] = acc[t][0];
    red[warp][g][8 * t + 2 * q + 1] = acc[t][1];
    red[warp][g + 8][8 * t + 2 * q] = acc[t][2];
    red[warp][g + 8][8 * t + 2 * q + 1] = acc[t][3];
  }
  __syncthreads();
  for (int e = threadIdx.x; e < 16 * R; e += 128) {
    const int row = e / R, col = e % R;
    const int64_t m = m0 + row;
    if (m >= M) continue;
    const float v = red[0][row][col] + red[1][row][col] + red[2][row][col] + red[3][row][col];
    partial[(static_cast<int64_t>(blockIdx.y) * M + m) * R + col] = v;
  }
}

__global__ void lora_rowproj_finish_kernel(const float* __restrict__ partial, int slices,
                                           int64_t M, int R, __nv_bfloat16* __restrict__ out_pad,
                                           __nv_bfloat16* __restrict__ out_dense) {
  pdl_launch_dependents();
  pdl_wait();  // inputs are the previous kernels' outputs
  const int64_t total = M * R;
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total;
       e += (int64_t)gridDim.x * blockDim.x) {
    float s = 0.f;
    for (int sl = 0; sl < slices; ++sl) s += partial[sl * total + e];
    const int64_t m = e / R, j = e % R;
    const __nv_bfloat16 v = __float2bfloat16_rn(s);
    out_pad[m * 64 + j] = v;
    if (out_dense) out_dense[e] = v;
  }
}

// Partial row reduction:  partial[chunk][j][d] = sum_{m in chunk} p[m][j0+j] * in[m][d]
// for a 16-wide group of adapter columns j0 = 16*blockIdx.z, one 256-column
// tile of D per CTA, on the tensor cores: per 16-row step,
// D[j][d] += P^T[j][m] . X[m][d] with mma.sync m16n8k16 (j = the 16 adapter
// columns, m = the reduced rows, d = 8 columns per n-tile).  Both operands
// are staged in shared memory 32 rows at a time (cp.async double buffer,
// rows past the chunk zero-filled) and read with ldmatrix.trans, which hands
// each thread the pairs along m the fragments need.  Warp w owns columns
// [32w, 32w + 32) of the 256-column tile, so no cross-warp reduction: every
// output is one warp's sum over the chunk's rows in order (deterministic).
// x rows: 512 B, 16-byte chunk c of row r stored at c ^ (r & 7); p rows: 32 B,
// half h of row r at h ^ ((r >> 2) & 1) -- both conflict-free for ldmatrix.
__device__ __forceinline__ void cp16_zfill(uint32_t dst, const void* src, uint32_t bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void ldsm4_trans(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                            uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

constexpr int kCpRows = 32;  // rows per staged tile

__global__ void __launch_bounds__(256) lora_colproj_mma_kernel(
    const __nv_bfloat16* __restrict__ p_pad, int64_t ld_p, const __nv_bfloat16* __restrict__ in,
    int64_t ld, int64_t M, int64_t D, int64_t rows_per_chunk, int R, float* __restrict__ partial) {
  pdl_launch_dependents();
  pdl_wait();  // inputs are the previous kernels' outputs
  __shared__ __align__(128) uint8_t xs[2][kCpRows * 512];
  __shared__ __align__(128) uint8_t ps[2][kCpRows * 32];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, q = lane & 3;
  const int64_t dt0 = static_cast<int64_t>(blockIdx.x) * 256;
  const int64_t chunk = blockIdx.y;
  const int j0 = blockIdx.z * 16;
  const int64_t mb = chunk * rows_per_chunk;
  const int64_t me = mb + rows_per_chunk < M ? mb + rows_per_chunk : M;

  auto load_tile = [&](int64_t mt, int buf) {
    const uint32_t xb = smem_u32(xs[buf]), pb = smem_u32(ps[buf]);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int c = tid + 256 * i, row = c >> 5, cc = c & 31;
      const int64_t m = mt + row, d = dt0 + cc * 8;
      const bool ok = m < me && d < D;
      cp16_zfill(xb + row * 512 + ((cc ^ (row & 7)) << 4), ok ? in + m * ld + d : in, ok ? 16u : 0u);
    }
    if (tid < 2 * kCpRows) {
      const int row = tid >> 1, h = tid & 1;
      const int64_t m = mt + row;
      const bool ok = m < me;
      cp16_zfill(pb + row * 32 + ((h ^ ((row >> 2) & 1)) << 4), ok ? p_pad + m * ld_p + j0 + 8 * h : p_pad,
                 ok ? 16u : 0u);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };

  float acc[4][4];
#pragma unroll
  for (int nt = 0; nt < 4; ++nt)
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[nt][e] = 0.f;

  const int mat = lane >> 3, r8 = lane & 7;
  int buf = 0;
  if (mb < me) load_tile(mb, 0);
  for (int64_t mt = mb; mt < me; mt += kCpRows, buf ^= 1) {
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    __syncthreads();  // tile mt visible; every warp is done with the other buffer
    if (mt + kCpRows < me) load_tile(mt + kCpRows, buf ^ 1);
    const uint32_t xb = smem_u32(xs[buf]), pb = smem_u32(ps[buf]);
#pragma unroll
    for (int ks = 0; ks < kCpRows / 16; ++ks) {
      uint32_t a0, a1, a2, a3;
      {
        // A = P^T: matrices (m 0-7 | 8-15 of the step) x (j 0-7 | 8-15)
        const int row = ks * 16 + (mat >> 1) * 8 + r8, h = mat & 1;
        ldsm4_trans(pb + row * 32 + ((h ^ ((row >> 2) & 1)) << 4), a0, a1, a2, a3);
      }
      uint32_t b[4][2];
#pragma unroll
      for (int np = 0; np < 2; ++np) {
        // B = X: matrices (m 0-7 | 8-15) x (n-tiles 2np, 2np + 1)
        const int row = ks * 16 + (mat & 1) * 8 + r8;
        const int cc = 4 * warp + 2 * np + (mat >> 1);
        ldsm4_trans(xb + row * 512 + ((cc ^ (row & 7)) << 4), b[2 * np][0], b[2 * np][1],
                    b[2 * np + 1][0], b[2 * np + 1][1]);
      }
#pragma unroll
      for (int nt = 0; nt < 4; ++nt) mma_bf16_16816(acc[nt], a0, a1, a2, a3, b[nt][0], b[nt][1]);
    }
  }
  // partial[chunk][j0 + j][d]: rows g / g + 8, columns 2q, 2q + 1 of each n-tile
#pragma unroll
  for (int nt = 0; nt < 4; ++nt) {
    const int64_t d = dt0 + 32 * warp + 8 * nt + 2 * q;
    if (d < D) {
      *reinterpret_cast<float2*>(partial + (chunk * R + j0 + g) * D + d) = make_float2(acc[nt][0], acc[nt][1]);
      *reinterpret_cast<float2*>(partial + (chunk * R + j0 + g + 8) * D + d) =
          make_float2(acc[nt][2], acc[nt][3]);
    }
  }
}

// res = (accumulate ? res : 0) + scale * sum_chunks partial, chunks in order.
__global__ void lora_colproj_finish_kernel(const float* __restrict__ partial, int64_t nchunks,
                                           int R, int64_t D, float scale, float* __restrict__ res,
                                           int layout, int accumulate) {
  pdl_launch_dependents();
  pdl_wait();  // inputs are the previous kernels' outputs
  const int64_t total = static_cast<int64_t>(R) * D;
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total;
       e += (int64_t)gridDim.x * blockDim.x) {
    float s = 0.f;
    for (int64_t c = 0; c < nchunks; ++c) s += partial[c * total + e];
    const int64_t j = e / D, d = e % D;
    const int64_t o = layout == 0 ? e : d * R + j;
    const float v = scale * s;
    res[o] = accumulate ? res[o] + v : v;
  }
}

// out[i][j] = bf16(scale * in(i, j)), pitch 64; in(i,j) = in[i*r + j] or, when
// transpose_in, in[j*rows + i].  Columns r..63 are zeroed.
__global__ void pad_lora_weight_kernel(const float* __restrict__ in, int64_t rows, int r,
                                       float scale, int transpose_in,
                                       __nv_bfloat16* __restrict__ out) {
  pdl_launch_dependents();
  pdl_wait();  // inputs are the previous kernels' outputs
  const int64_t total = rows * 64;
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total;
       e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t i = e >> 6;
    const int j = static_cast<int>(e & 63);
    float v = 0.f;
    if (j < r) v = scale * (transpose_in ? in[j * rows + i] : in[i * r + j]);
    out[e] = __float2bfloat16_rn(v);
  }
}

__global__ void f32_to_bf16_kernel(const float* __restrict__ in, int64_t n,
                                   __nv_bfloat16* __restrict__ out) {
  pdl_launch_dependents();
  pdl_wait();  // inputs are the previous kernels' outputs
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < n;
       e += (int64_t)gridDim.x * blockDim.x)
    out[e] = __float2bfloat16_rn(in[e]);
}

// out[j][i] = bf16(in[i][j]) for in fp32 [rows, cols].
__global__ void f32_to_bf16_t_kernel(const float* __restrict__ in, int64_t rows, int cols,
                                     __nv_bfloat16* __restrict__ out) {
  pdl_launch_dependents();
  pdl_wait();  // inputs are the previous kernels' outputs
  const int64_t total = rows * cols;
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total;
       e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t j = e / rows, i = e % rows;  // output index e = j*rows + i
    out[e] = __float2bfloat16_rn(in[i * cols + j]);
  }
}

int grid_for(int64_t n, int threads, int num_sms) {
  int64_t b = (n + threads - 1) / threads;
  int64_t cap = static_cast<int64_t>(num_sms) * 16;
  return static_cast<int>(b < cap ? (b > 0 ? b : 1) : cap);
}

void colproj_geometry(int64_t M, int64_t D, int num_sms, int64_t* rows_per_chunk,
                      int64_t* nchunks) {
  const int64_t dtiles = (D + 255) / 256;
  int64_t want = (2 * static_cast<int64_t>(num_sms) + dtiles - 1) / dtiles;
  if (want < 1) want = 1;
  int64_t rpc = (M + want - 1) / want;
  rpc = ((rpc + 7) / 8) * 8;
  if (rpc < 8) rpc = 8;
  *rows_per_chunk = rpc;
  *nchunks = (M + rpc - 1) / rpc;
}

// Partial T[m][j] = sum_k x[m,k] * bf16(A[j,k]) over one 64-column group per
// CTA, for the decode / verify row counts: CTA c stages columns
// [64c, 64c+64) of A (rounded to bf16, as the reference's bf16 lora_A
// projection under autocast does: fitllm/qlora.py:74-83,
// fitllm/forward.py:254-257) and of x in shared memory (row pitch 129 floats:
// conflict-free), splits each (m, j) dot product over a group of `tp` lanes
// closed by a fixed butterfly, and writes part[c][m][j] (fp32).  The
// finishing kernel sums the groups in order.
//
// Launch order (programmatic dependent launch): the decode GEMV, then this
// kernel, then the finishing kernel.  The GEMV waits for its own predecessor
// before letting this kernel launch, so x is complete and this kernel reads it
// without waiting, on the SMs the GEMV leaves free; CTA 0 waits for the GEMV
// before exiting, so the finishing kernel's wait on this grid covers the
// GEMV's partial sums too.
constexpr int kTCols = 64;

// blockIdx.y picks one of up to three (A, rank, partials) jobs on the same x
// (the LoRA projections of a grouped q/k/v call share one launch).
struct LoraTJobs {
  const float* a[3];
  float* part[3];
  int r[3];
  int tp[3];
};

__global__ void __launch_bounds__(256)
    lora_t_kernel(const __nv_bfloat16* __restrict__ x, int M, int K, LoraTJobs tj) {
  extern __shared__ float s_lt[];
  pdl_launch_dependents();
  const int jy = blockIdx.y;
  const float* __restrict__ a = jy == 0 ? tj.a[0] : jy == 1 ? tj.a[1] : tj.a[2];
  float* __restrict__ part = jy == 0 ? tj.part[0] : jy == 1 ? tj.part[1] : tj.part[2];
  const int r = jy == 0 ? tj.r[0] : jy == 1 ? tj.r[1] : tj.r[2];
  const int tp = jy == 0 ? tj.tp[0] : jy == 1 ? tj.tp[1] : tj.tp[2];
  constexpr int pitch = kTCols + 1;
  const int c0 = blockIdx.x * kTCols;
  float* as = s_lt;
  float* xs = s_lt + r * pitch;
  // staging: 16-byte loads, all issued before the shared-memory stores
  {
    constexpr int per_row4 = kTCols / 4;  // float4 per A row
    const int na = r * per_row4;
    for (int b = threadIdx.x; b < na; b += 4 * 256) {
      float4 v[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int i = b + u * 256;
        if (i < na)
          v[u] = __ldg(reinterpret_cast<const float4*>(a + static_cast<int64_t>(i / per_row4) * K + c0) +
                       i % per_row4);
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int i = b + u * 256;
        if (i < na) {
          float* d = as + (i / per_row4) * pitch + 4 * (i % per_row4);
          d[0] = __bfloat162float(__float2bfloat16_rn(v[u].x));
          d[1] = __bfloat162float(__float2bfloat16_rn(v[u].y));
          d[2] = __bfloat162float(__float2bfloat16_rn(v[u].z));
          d[3] = __bfloat162float(__float2bfloat16_rn(v[u].w));
        }
      }
    }
    constexpr int per_row8 = kTCols / 8;  // 8 bf16 per uint4
    for (int i = threadIdx.x; i < M * per_row8; i += 256) {
      const uint4 v = __ldg(reinterpret_cast<const uint4*>(x + static_cast<int64_t>(i / per_row8) * K + c0) +
                            i % per_row8);
      float* d = xs + (i / per_row8) * pitch + 8 * (i % per_row8);
      const uint32_t w4[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        d[2 * h] = __uint_as_float(w4[h] << 16);
        d[2 * h + 1] = __uint_as_float(w4[h] & 0xFFFF0000u);
      }
    }
  }
  __syncthreads();
  // pair pi = (m, j) handled by lanes [sub*tp, sub*tp + tp) of a group; tp | 32
  const int groups = blockDim.x / tp, sub = threadIdx.x % tp;
  const int kper = kTCols / tp;
  for (int base = 0; base < M * r; base += groups) {
    const int pi = base + threadIdx.x / tp;
    float s = 0.f;
    if (pi < M * r) {
      const int m = pi / r, j = pi % r;
      const float* xr = xs + m * pitch + sub * kper;
      const float* ar = as + j * pitch + sub * kper;
      for (int k = 0; k < kper; ++k) s = fmaf(xr[k], ar[k], s);
    }
    for (int sh = tp / 2; sh > 0; sh >>= 1) s += __shfl_xor_sync(0xffffffffu, s, sh);
    if (sub == 0 && pi < M * r) part[static_cast<int64_t>(blockIdx.x) * M * r + pi] = s;
  }
  if (blockIdx.x == 0) pdl_wait();  // this grid completes after the GEMV launched before it
}

}  // namespace

int launch_lora_rowproj(const void* in, int64_t ld_in, int64_t M, int64_t D, const void* wt_bf16,
                        int r, void* out_pad, void* out_dense, cudaStream_t st, int num_sms) {
  (void)num_sms;
  const int grid = static_cast<int>((M + 15) / 16);
  auto i = static_cast<const __nv_bfloat16*>(in);
  auto w = static_cast<const __nv_bfloat16*>(wt_bf16);
  auto op = static_cast<__nv_bfloat16*>(out_pad);
  auto od = static_cast<__nv_bfloat16*>(out_dense);
  switch (r) {
    case 16: launch_pdl(lora_rowproj_kernel<16>, dim3(grid), dim3(128), 0, st, i, ld_in, M, D, w, op, od); note_launch(); break;
    case 32: launch_pdl(lora_rowproj_kernel<32>, dim3(grid), dim3(128), 0, st, i, ld_in, M, D, w, op, od); note_launch(); break;
    case 48: launch_pdl(lora_rowproj_kernel<48>, dim3(grid), dim3(128), 0, st, i, ld_in, M, D, w, op, od); note_launch(); break;
    case 64: launch_pdl(lora_rowproj_kernel<64>, dim3(grid), dim3(128), 0, st, i, ld_in, M, D, w, op, od); note_launch(); break;
    default: return FITQ_ERR_UNSUPPORTED;
  }
  return launch_result();
}

size_t lora_rowproj_small_workspace(int64_t M, int64_t D, int r) {
  const int64_t slices = (D + kRowprojSlice - 1) / kRowprojSlice;
  return static_cast<size_t>(slices * M * r) * sizeof(float);
}

int launch_lora_rowproj_small(const void* in, int64_t ld_in, int64_t M, int64_t D,
                              const void* wt_bf16, int r, float* partial_ws, void* out_pad,
                              void* out_dense, cudaStream_t st) {
  const int64_t slices = (D + kRowprojSlice - 1) / kRowprojSlice;
  dim3 grid(static_cast<unsigned>((M + 15) / 16), static_cast<unsigned>(slices));
  auto i = static_cast<const __nv_bfloat16*>(in);
  auto w = static_cast<const __nv_bfloat16*>(wt_bf16);
  switch (r) {
    case 16: launch_pdl(lora_rowproj_split_kernel<16>, grid, dim3(128), 0, st, i, ld_in, M, D, w, partial_ws); break;
    case 32: launch_pdl(lora_rowproj_split_kernel<32>, grid, dim3(128), 0, st, i, ld_in, M, D, w, partial_ws); break;
    case 48: launch_pdl(lora_rowproj_split_kernel<48>, grid, dim3(128), 0, st, i, ld_in, M, D, w, partial_ws); break;
    case 64: launch_pdl(lora_rowproj_split_kernel<64>, grid, dim3(128), 0, st, i, ld_in, M, D, w, partial_ws); break;
    default: return FITQ_ERR_UNSUPPORTED;
  }
  note_launch();
  launch_pdl(lora_rowproj_finish_kernel, dim3(grid_for(M * r, 256, 148)), dim3(256), 0, st,
             static_cast<const float*>(partial_ws), static_cast<int>(slices), M, r,
             static_cast<__nv_bfloat16*>(out_pad), static_cast<__nv_bfloat16*>(out_dense));
  note_launch();
  return launch_result();
}

size_t lora_t_workspace(int64_t M, int64_t K, int r) {
  return static_cast<size_t>((K / kTCols) * M * r) * sizeof(float);
}

int lora_t_groups(int64_t K) { return static_cast<int>(K / kTCols); }

int launch_lora_t_multi(const void* x, int64_t M, int64_t K, const float* const* a, const int* r,
                        float* const* part_ws, int jobs, cudaStream_t st) {
  if (K % kTCols != 0 || M < 1 || M > 64 || jobs < 1 || jobs > 3) return FITQ_ERR_UNSUPPORTED;
  LoraTJobs tj{};
  int r_max = 0;
  for (int j = 0; j < 3; ++j) {
    const int jj = j < jobs ? j : jobs - 1;
    if (r[jj] < 1 || r[jj] > 64 || r[jj] % 4 != 0) return FITQ_ERR_UNSUPPORTED;
    tj.a[j] = a[jj];
    tj.part[j] = part_ws[jj];
    tj.r[j] = r[jj];
    int tp = 32;  // lanes per (m, j) dot product: fill the 256 threads
    while (tp > 1 && static_cast<int64_t>(256 / tp) < M * r[jj]) tp >>= 1;
    tj.tp[j] = tp;
    r_max = r[jj] > r_max ? r[jj] : r_max;
  }
  const size_t smem = static_cast<size_t>(r_max + M) * (kTCols + 1) * sizeof(float);
  if (!set_smem_limit(lora_t_kernel, (64 + 64) * (kTCols + 1) * static_cast<int>(sizeof(float))))
    return FITQ_ERR_CUDA;
  const cudaError_t e = launch_pdl(lora_t_kernel, dim3(static_cast<unsigned>(K / kTCols), jobs), dim3(256),
                                   smem, st, static_cast<const __nv_bfloat16*>(x), static_cast<int>(M),
                                   static_cast<int>(K), tj);
  note_launch();
  return e == cudaSuccess ? FITQ_OK : FITQ_ERR_CUDA;
}

int launch_lora_t(const void* x, int64_t M, int64_t K, const float* a, int r, float* part_ws,
                  cudaStream_t st) {
  return launch_lora_t_multi(x, M, K, &a, &r, &part_ws, 1, st);
}

size_t lora_colproj_workspace(int64_t M, int64_t D, int r, int num_sms) {
  int64_t rpc, nch;
  colproj_geometry(M, D, num_sms, &rpc, &nch);
  return static_cast<size_t>(nch) * r * D * sizeof(float);
}

int launch_lora_colproj(const void* p_pad, int64_t ld_p, const void* in, int64_t ld_in, int64_t M,
                        int64_t D, int r, float scale, float* res, int layout, int accumulate,
                        float* partial_ws, cudaStream_t st, int num_sms) {
  int64_t rpc, nch;
  colproj_geometry(M, D, num_sms, &rpc, &nch);
  dim3 grid(static_cast<unsigned>((D + 255) / 256), static_cast<unsigned>(nch),
            static_cast<unsigned>(r / 16));
  launch_pdl(lora_colproj_mma_kernel, dim3(grid), dim3(256), 0, st,
             static_cast<const __nv_bfloat16*>(p_pad), ld_p, static_cast<const __nv_bfloat16*>(in),
             ld_in, M, D, rpc, r, partial_ws);
  note_launch();
  launch_pdl(lora_colproj_finish_kernel, dim3(grid_for(static_cast<int64_t>(r) * D, 256, num_sms)),
             dim3(256), 0, st, static_cast<const float*>(partial_ws), nch, r, D, scale, res, layout,
             accumulate);
  note_launch();
  return launch_result();
}

int launch_pad_lora_weight(const float* in, int64_t rows, int r, float scale, int transpose_in,
                           void* out_pad, cudaStream_t st) {
  launch_pdl(pad_lora_weight_kernel, dim3(grid_for(rows * 64, 256, 148)), dim3(256), 0, st, in, rows, r,
             scale, transpose_in, static_cast<__nv_bfloat16*>(out_pad));
  note_launch();
  return launch_result();
}

int launch_f32_to_bf16_t(const float* in, int64_t rows, int cols, void* out, cudaStream_t st) {
  launch_pdl(f32_to_bf16_t_kernel, dim3(grid_for(rows * cols, 256, 148)), dim3(256), 0, st, in, rows,
             cols, static_cast<__nv_bfloat16*>(out));
  note_launch();
  return launch_result();
}

int launch_f32_to_bf16(const float* in, int64_t n, void* out, cudaStream_t st) {
  launch_pdl(f32_to_bf16_kernel, dim3(grid_for(n, 256, 148)), dim3(256), 0, st, in, n,
             static_cast<__nv_bfloat16*>(out));
  note_launch();
  return launch_result();
}

}  // namespace fitq
