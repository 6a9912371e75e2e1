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

__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
      "{%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
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

// ---------------------------------------------------------------------------
// Decode kernel for M <= 8 tokens (one n8 token tile), one launch per GEMV.
//
// A CTA owns one K slice of kw*4 blocks and a strided set of 16-row tiles;
// warp (rg, p) = (warp / kw, warp % kw) covers blocks [4p, 4p+4) of the slice
// for every rtg-th tile of the CTA.  Because a warp's K range never changes,
// its x fragments live in registers for the whole kernel.
//
// HBM only runs near its peak with 64-100 KB of reads in flight per SM, more
// than registers can hold next to the decode, so each warp streams its own
// tiles (16 rows x 128 bytes) into a private 3-stage shared-memory ring with
// 16-byte cp.async copies: two tiles in flight while the third is decoded,
// with no cross-warp synchronisation (a warp only reads what it copied).
// Within a staged row, 16-byte chunk k is stored at chunk k ^ 2*(row & 3),
// which makes the 8-byte fragment reads conflict-free without padding.  The
// absmax codes and nested scales (8 bytes per row and tile) ride a small
// register ring two tiles ahead; each lane decodes the absmax of one (row,
// block) pair of the tile and the warp shares them through shared memory.
//
// The code table sits on a 64 KB boundary of the CTA's shared window, so one
// prmt of (packed byte, lane base) yields the complete shared address of a
// lane's bf16 pair and the lookup is a single ld.shared.  The nested absmax
// map lives in the unused upper half of each 256-byte entry (8 copies, one per
// lane row g): an absmax costs one prmt + one ld.shared + the reference's two
// rounded fp32 ops.  The kw partial sums of a tile are combined through shared
// memory every second round of 3 tiles, in k order (deterministic), by the kw
// warps of the row group alone, which meet on a named barrier of their own.
//
// Epilogue: with one K slice and no LoRA the sums go straight to y (+ bias +
// y_add, bf16) in this kernel.  Otherwise each slice writes fp32 partials
// partial[slice][m][n] and gemv_dec_finish_kernel sums them in slice order
// (deterministic) and adds scale * T.B^T + bias + y_add; the LoRA T kernel
// runs between the two, on the SMs this grid leaves free, while the weights
// stream.
//
// Launched with programmatic dependent launch: before griddepcontrol.wait the
// kernel only prefetches its first weight tiles into L2 (safe even if the
// predecessor writes them: L2 is the point of coherence), so the DRAM latency
// of the stream's start overlaps the predecessor's tail.
// ---------------------------------------------------------------------------
constexpr int kDecKB = 4;                      // blocks per warp and tile
constexpr int kDecRing = 3;                    // ring stages per warp
constexpr int kDecDepth = kDecRing - 1;        // tiles in flight ahead of the decoded one
constexpr int kDecStage = 16 * 128;            // one staged tile (16 rows x 128 bytes, swizzled)
constexpr int kDecSmem = 232448;               // the whole 227 KB: table alignment slack + table + ring + reduction

struct Gemv8Plan {
  int kw, rtg, cs, slices;
  int lkw, lrtg, lqn;  // log2 of kw, rtg and of the token lanes stored per row (qn)
};

template <bool NESTED>
struct ScaleBuf {
  uint32_t ca, cb;  // absmax codes of the 4 blocks of rows a = 16t+g and b = a+8
  float na, nb;     // nested absmax (a 4-aligned block range stays in one 256-block group)
  float4 fa, fb;    // fp32 absmax when not double-quantised
};

__device__ __forceinline__ uint64_t evict_first_policy() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, uint64_t pol) {
  asm volatile("cp.async.cg.shared.global.L2::cache_hint [%0], [%1], 16, %2;" ::"r"(dst), "l"(src),
               "l"(pol)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void prefetch_l2(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

__device__ __forceinline__ uint2 lds64(uint32_t addr) {
  uint2 v;
  asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(addr));
  return v;
}

__device__ __forceinline__ float4 lds128f(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(addr)
               : "memory");
  return v;
}

__device__ __forceinline__ void sts32(uint32_t addr, float v) {
  asm volatile("st.shared.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}

// Shared address of byte J of v in the 64 KB-aligned table: bits 16..31 and
// 0..7 from base (table | lane offset), bits 8..15 = the byte.
template <int J>
__device__ __forceinline__ uint32_t tbl_addr(uint32_t v, uint32_t base) {
  uint32_t r;
  constexpr uint32_t sel = 0x7600u | (static_cast<uint32_t>(J) << 4) | 4u;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(v), "r"(base), "n"(sel));
  return r;
}

template <int J>
__device__ __forceinline__ uint32_t tbl_u32(uint32_t v, uint32_t base) {
  uint32_t r;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(r) : "r"(tbl_addr<J>(v, base)));
  return r;
}

// Same with the byte chosen at run time (sel = 0x7604 | byte << 4).
__device__ __forceinline__ float tbl_f32_sel(uint32_t v, uint32_t base, uint32_t sel) {
  uint32_t a, r;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(a) : "r"(v), "r"(base), "r"(sel));
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(r) : "r"(a));
  return __uint_as_float(r);
}

template <bool NESTED>
__device__ __forceinline__ void load_scales(ScaleBuf<NESTED>& b, const Nf4Args& w, int fa,
                                            int nblk8) {
  if (NESTED) {
    b.ca = __ldg(reinterpret_cast<const uint32_t*>(w.absmax_code + fa));
    b.cb = __ldg(reinterpret_cast<const uint32_t*>(w.absmax_code + fa + nblk8));
    b.na = __ldg(w.nested_absmax + (fa >> 8));
    b.nb = __ldg(w.nested_absmax + ((fa + nblk8) >> 8));
  } else {
    b.fa = __ldg(reinterpret_cast<const float4*>(w.absmax_f32 + fa));
    b.fb = __ldg(reinterpret_cast<const float4*>(w.absmax_f32 + fa + nblk8));
  }
}

__device__ __forceinline__ void mma16816_zc(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                            uint32_t a3, uint32_t b0, uint32_t b1) {
  const float z = 0.f;
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
      "{%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, {%10, %10, %10, %10};"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(z));
}

// One 16x64 block: 4 MMAs over the decoded A fragments, scaled per row.
__device__ __forceinline__ void block_mma(float4& acc, uint2 wa, uint2 wb, uint4 x0, uint4 x1,
                                          uint32_t lb, float am_a, float am_b) {
  float t[4];
  // byte 2i of the lane's 8 bytes -> cols 16q+4i+{0,1}, byte 2i+1 -> cols 16q+4i+{2,3}
  mma16816_zc(t, tbl_u32<0>(wa.x, lb), tbl_u32<0>(wb.x, lb), tbl_u32<1>(wa.x, lb),
              tbl_u32<1>(wb.x, lb), x0.x, x0.y);
  mma16816(t, tbl_u32<2>(wa.x, lb), tbl_u32<2>(wb.x, lb), tbl_u32<3>(wa.x, lb),
           tbl_u32<3>(wb.x, lb), x0.z, x0.w);
  mma16816(t, tbl_u32<0>(wa.y, lb), tbl_u32<0>(wb.y, lb), tbl_u32<1>(wa.y, lb),
           tbl_u32<1>(wb.y, lb), x1.x, x1.y);
  mma16816(t, tbl_u32<2>(wa.y, lb), tbl_u32<2>(wb.y, lb), tbl_u32<3>(wa.y, lb),
           tbl_u32<3>(wb.y, lb), x1.z, x1.w);
  acc.x = fmaf(t[0], am_a, acc.x);
  acc.y = fmaf(t[1], am_a, acc.y);
  acc.z = fmaf(t[2], am_b, acc.z);
  acc.w = fmaf(t[3], am_b, acc.w);
}

// frag[c]: the lane's fragment offset of block c of row g inside a stage
// (row g + 8 is 1024 bytes further, same swizzle); am_a / am_b: the absmax of
// blocks 0..3 of rows g and g + 8.
template <int C>
__device__ __forceinline__ void stage_block(float4& acc, uint32_t stage,
                                            const uint32_t (&frag)[kDecKB], float4 am_a,
                                            float4 am_b, const uint4 (&xr)[kDecKB][2],
                                            uint32_t lb) {
  const uint32_t a = stage + frag[C];
  const uint2 wa = lds64(a), wb = lds64(a + 8 * 128);
  const float sa = C == 0 ? am_a.x : C == 1 ? am_a.y : C == 2 ? am_a.z : am_a.w;
  const float sb = C == 0 ? am_b.x : C == 1 ? am_b.y : C == 2 ? am_b.z : am_b.w;
  block_mma(acc, wa, wb, xr[C][0], xr[C][1], lb, sa, sb);
}

// Partial sums of one staged tile: lane (g, q) returns rows (g, g+8) x tokens (2q, 2q+1).
__device__ __forceinline__ float4 compute_tile(uint32_t stage, const uint32_t (&frag)[kDecKB],
                                               float4 am_a, float4 am_b,
                                               const uint4 (&xr)[kDecKB][2], uint32_t lb) {
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  stage_block<0>(acc, stage, frag, am_a, am_b, xr, lb);
  stage_block<1>(acc, stage, frag, am_a, am_b, xr, lb);
  stage_block<2>(acc, stage, frag, am_a, am_b, xr, lb);
  stage_block<3>(acc, stage, frag, am_a, am_b, xr, lb);
  return acc;
}

// Absmax of blocks 0..3 of rows g and g + 8 of the tile.  Double-quantised:
// lane (g, q) decodes block q of both rows and the warp exchanges them through
// its 256-byte scale area (rows x blocks, fp32).
template <bool NESTED>
__device__ __forceinline__ void tile_scales(const ScaleBuf<NESTED>& b, uint32_t nq_base,
                                            uint32_t sel_q, float offset, uint32_t sc_w,
                                            uint32_t sc_lane, int g, float4& am_a,
                                            float4& am_b) {
  if (NESTED) {
    sts32(sc_lane, __fadd_rn(__fmul_rn(tbl_f32_sel(b.ca, nq_base, sel_q), b.na), offset));
    sts32(sc_lane + 128, __fadd_rn(__fmul_rn(tbl_f32_sel(b.cb, nq_base, sel_q), b.nb), offset));
    __syncwarp();
    am_a = lds128f(sc_w + 16 * g);
    am_b = lds128f(sc_w + 128 + 16 * g);
  } else {
    am_a = b.fa;
    am_b = b.fb;
  }
}

// y[tk, n] = bf16(s + scale * T[tk].B[n] + bias[n] + y_add[tk, n]); tl: row tk of
// T as fp32 (bf16-rounded values), null when rank == 0.
__device__ __forceinline__ float dec_value(const GemvEpilogue& o, const float* tl, int N, int tk,
                                           int n, float s) {
  if (o.rank > 0) {
    const float4* bl = reinterpret_cast<const float4*>(o.lora_b + static_cast<int64_t>(n) * o.rank);
    float l = 0.f;
    for (int j = 0; j < o.rank; j += 4) {
      const float4 b = __ldg(bl + j / 4);
      l = fmaf(tl[j], b.x, l);
      l = fmaf(tl[j + 1], b.y, l);
      l = fmaf(tl[j + 2], b.z, l);
      l = fmaf(tl[j + 3], b.w, l);
    }
    s += o.scale * l;
  }
  const int64_t e = static_cast<int64_t>(tk) * N + n;
  if (o.bias) s += __bfloat162float(static_cast<const __nv_bfloat16*>(o.bias)[n]);
  if (o.y_add) s += __bfloat162float(static_cast<const __nv_bfloat16*>(o.y_add)[e]);
  return s;
}

__device__ __forceinline__ void dec_store(const GemvEpilogue& o, const float* tl, int N, int tk,
                                          int n, float s) {
  static_cast<__nv_bfloat16*>(o.y)[static_cast<int64_t>(tk) * N + n] =
      __float2bfloat16_rn(dec_value(o, tl, N, tk, n, s));
}

// Staged row r (r & 3 == lane >> 3 for every copy of a lane): 16-byte chunk k
// at chunk k ^ 2*(r & 3) of the 128-byte row.
__device__ __forceinline__ uint32_t dst_lane_of(int lane) {
  return static_cast<uint32_t>((lane >> 3) * 128 + 16 * ((lane & 7) ^ (2 * (lane >> 3))));
}

// Which weight of a grouped launch tile t belongs to (DecJobs in kernels.cuh).
__device__ __forceinline__ int dec_job(const DecJobs& jb, int t) {
  return (t >= jb.tile0[1]) + (t >= jb.tile0[2]);
}

template <bool NESTED>
__global__ void __launch_bounds__(kThreads, 1)
    nf4_gemv_dec_kernel(DecJobs jb, const __nv_bfloat16* __restrict__ x, int M, Gemv8Plan pl,
                        GemvEpilogue out) {
  constexpr int R = kDecRing, D = kDecDepth;
  const Nf4Args& w = jb.w[0];  // K, code tables (shared by every weight of the launch)
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, q = lane & 3;
  const int K = static_cast<int>(w.k_in);
  const int nblk = K / 64, T = jb.tile0[3];
  const int qn = 1 << pl.lqn;  // token lanes q < qn hold tokens 2q, 2q+1 < 2*qn >= M

  const int slice = blockIdx.x / pl.cs, j = blockIdx.x % pl.cs;
  const int p = warp & (pl.kw - 1), rg = warp >> pl.lkw;
  const int b0 = (slice * pl.kw + p) * kDecKB;  // first block of this warp's K range
  // this warp's tiles: t_u = j + cs * (rg + rtg * u)
  const int tstride = pl.cs << pl.lrtg;
  const int t0 = j + pl.cs * rg;
  const int n_u = t0 < T ? (T - 1 - t0) / tstride + 1 : 0;

  // Before the dependency wait: L2 prefetch of this warp's first tiles only.
  if (lane < 16) {
    for (int u = 0; u < kDecDepth && u < n_u; ++u) {
      const int t = t0 + u * tstride, jj = dec_job(jb, t);
      prefetch_l2(jb.w[jj].packed +
                      (static_cast<int64_t>(16 * (t - jb.tile0[jj]) + lane) * nblk + b0) * 32,
                  kDecKB * 32);
    }
  }
  // Wait first, then let dependents launch: a LoRA T kernel launched right
  // behind this one reads x without waiting (see launch_lora_t).
  pdl_wait();
  pdl_launch_dependents();

  // Shared layout: [slack below the 64 KB boundary][table 64 KB][rest].  Ring
  // stages fill the slack first, then the rest; the reduction area and the
  // per-warp scale areas follow.
  const uint32_t sbase = smem_u32(g_gemv_smem);
  const uint32_t tbl = (sbase + 0xFFFFu) & ~0xFFFFu;
  const int n_slack = static_cast<int>((tbl - sbase) / kDecStage);
  const uint32_t after = tbl + kTableBytes;
  const int n_ring = kWarps * R;
  const uint32_t red_addr =
      after + static_cast<uint32_t>(n_ring > n_slack ? n_ring - n_slack : 0) * kDecStage;
  float4* const red = reinterpret_cast<float4*>(g_gemv_smem + (red_addr - sbase));
  const int red_warp = 8 * qn;  // float4 slots per warp and tile
  // two rounds of reduction slots: the k-parts are summed every second round
  const uint32_t sc_addr = red_addr + static_cast<uint32_t>(2 * R * kWarps * 8 * 4 * 16);  // 256 B per warp

  // ring stages of this warp
  uint32_t stage[R];
#pragma unroll
  for (int s = 0; s < R; ++s) {
    const int i = warp * R + s;
    stage[s] = i < n_slack ? sbase + static_cast<uint32_t>(i) * kDecStage
                           : after + static_cast<uint32_t>(i - n_slack) * kDecStage;
  }

  const int n_u_max = j < T ? (T - 1 - j) / tstride + 1 : 0;  // row group 0 has the most
  const int rounds = (n_u_max + D) / R;
  const int nblk8 = 8 * nblk;
  // copies: lane covers 16 bytes (lane & 7) of rows (lane >> 3) + 4j, j = 0..3
  const int64_t row_bytes = K / 2;
  // tile u of this warp: its weight's copies and scales (flat block of row g)
  auto issue_tile = [&](uint32_t stg, ScaleBuf<NESTED>& sbuf, int u, uint64_t pol) {
    const int t = t0 + u * tstride, jj = dec_job(jb, t), tl = t - jb.tile0[jj];
    const uint8_t* src = jb.w[jj].packed + (static_cast<int64_t>(16 * tl + (lane >> 3)) * nblk + b0) * 32 +
                         16 * (lane & 7);
#pragma unroll
    for (int c = 0; c < 4; ++c) cp_async16(stg + dst_lane_of(lane) + c * 512, src + c * 4 * row_bytes, pol);
    load_scales(sbuf, jb.w[jj], (16 * tl + g) * nblk + b0, nblk8);
  };
  uint32_t frag[kDecKB];  // fragment reads: row g, bytes 32c + 8q, swizzled
#pragma unroll
  for (int c = 0; c < kDecKB; ++c)
    frag[c] = static_cast<uint32_t>(g * 128 + 32 * (c ^ (g & 3)) + 8 * q);
  const uint32_t lb = tbl | (static_cast<uint32_t>(lane) << 2);
  const uint32_t nq_base = tbl | (128u + (static_cast<uint32_t>(g) << 2));
  const uint32_t sel_q = 0x7604u | (static_cast<uint32_t>(q) << 4);  // byte q of a code word
  const uint32_t sc_w = sc_addr + static_cast<uint32_t>(warp) * 256u;
  const uint32_t sc_lane = sc_w + static_cast<uint32_t>(g * 16 + 4 * q);
  const uint64_t pol = evict_first_policy();

  // The first tiles' copies go out before the table fill and the x loads, so
  // their latency overlaps that setup.
  ScaleBuf<NESTED> sb[R];
#pragma unroll
  for (int d = 0; d < D; ++d) {
    if (d < n_u) issue_tile(stage[d], sb[d], d, pol);
    cp_async_commit();
  }
  // entry e (256 B): lanes' bf16 pairs {qm[e >> 4], qm[e & 15]} at 4l, nested map at 128 + 4g;
  // two threads per entry, 16-byte stores
  {
    uint4* table = reinterpret_cast<uint4*>(g_gemv_smem + (tbl - sbase));
    const int e = threadIdx.x >> 1, h = threadIdx.x & 1;
    const uint32_t v = pack_bf16x2(__ldg(w.quant_map + (e >> 4)), __ldg(w.quant_map + (e & 15)));
    const uint4 vv = make_uint4(v, v, v, v);
#pragma unroll
    for (int i = 0; i < 4; ++i) table[e * 16 + h * 4 + i] = vv;
    if (NESTED) {
      const uint32_t nv = __float_as_uint(__ldg(w.nested_quant_map + e));
      table[e * 16 + 8 + h] = make_uint4(nv, nv, nv, nv);
    }
    // One code table serves every weight of a grouped launch: their maps must hold the same values.
    for (int gg = 1; gg < jb.groups; ++gg) {
      bool same = true;
      if (threadIdx.x < 16) same = __ldg(jb.w[gg].quant_map + threadIdx.x) == __ldg(w.quant_map + threadIdx.x);
      if (NESTED && threadIdx.x < 256)
        same = same && __ldg(jb.w[gg].nested_quant_map + threadIdx.x) == __ldg(w.nested_quant_map + threadIdx.x);
      if (!same) report_device_error(jb.status, FITQ_ERR_UNSUPPORTED);
    }
  }

  uint4 xr[kDecKB][2];
#pragma unroll
  for (int c = 0; c < kDecKB; ++c) {
    if (g < M) {
      const uint4* xs = reinterpret_cast<const uint4*>(x + static_cast<int64_t>(g) * K +
                                                       (b0 + c) * 64 + 16 * q);
      xr[c][0] = __ldg(xs);
      xr[c][1] = __ldg(xs + 1);
    } else {
      xr[c][0] = make_uint4(0, 0, 0, 0);
      xr[c][1] = make_uint4(0, 0, 0, 0);
    }
  }

  __syncthreads();  // table ready

  // barrier of the kw warps of row group rg (a single warp needs none)
  auto group_sync = [&]() {
    if (pl.kw == 1) {
      __syncwarp();
    } else {
      asm volatile("bar.sync %0, %1;" ::"r"(1 + rg), "r"(pl.kw * 32) : "memory");
    }
  };

  for (int rd = 0; rd < rounds; ++rd) {
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const int u = rd * R + r;
      __syncwarp();  // every lane is done with the stage refilled below (decoded last step)
      if (u + D < n_u) issue_tile(stage[(r + D) % R], sb[(r + D) % R], u + D, pol);
      cp_async_commit();
      cp_async_wait<D>();  // this lane's copies of tile u have landed
      __syncwarp();        // ... and every other lane's
      float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
      if (u < n_u) {
        float4 am_a, am_b;
        const float offset = jb.groups > 1 ? jb.w[dec_job(jb, t0 + u * tstride)].offset : w.offset;
        tile_scales(sb[r], nq_base, sel_q, offset, sc_w, sc_lane, g, am_a, am_b);
        o = compute_tile(stage[r], frag, am_a, am_b, xr, lb);
      }
      if (q < qn) red[((r + R * (rd & 1)) * kWarps + warp) * red_warp + (g << pl.lqn) + q] = o;
    }
    if ((rd & 1) == 0 && rd + 1 < rounds) continue;  // reduce two rounds at once
    // Only the kw warps of this row group exchange partial sums: they meet on
    // their own named barrier (1 + rg), so row groups do not wait on each other.
    group_sync();
    // sum the kw parts of each tile of rounds rd0..rd in k order; slot f = (g*qn + q)*4 + component
    const int rd0 = rd & ~1;
    const int fbits = 5 + pl.lqn;
    const int outs = ((rd - rd0 + 1) * R) << fbits;
    const float* rf = reinterpret_cast<const float*>(red);
    for (int e = p * 32 + lane; e < outs; e += pl.kw * 32) {
      const int f = e & ((1 << fbits) - 1), r = e >> fbits;
      const int rgo = rg;
      const int ls = f >> 2, comp = f & 3;
      const int rr = (ls >> pl.lqn) + 8 * (comp >> 1);
      const int tk = 2 * (ls & (qn - 1)) + (comp & 1);
      const int t = j + pl.cs * (rgo + ((rd0 * R + r) << pl.lrtg));
      if (tk >= M || t >= T) continue;
      const float* srcf = rf + (((r * kWarps + (rgo << pl.lkw)) * red_warp) << 2) + f;
      float s = 0.f;
      for (int pp = 0; pp < pl.kw; ++pp) s += srcf[(pp * red_warp) << 2];
      const int jj = dec_job(jb, t);
      const int nj = static_cast<int>(jb.w[jj].n_out), row = (t - jb.tile0[jj]) * 16 + rr;
      if (jb.partial[jj] == nullptr) dec_store(out, nullptr, nj, tk, row, s);
      else jb.partial[jj][(static_cast<int64_t>(slice) * M + tk) * nj + row] = s;
    }
    group_sync();  // the group's reduction slots are rewritten from the next round on
  }
  cp_async_wait<0>();
}

// Finishing pass of the split-K decode / skinny GEMMs: y[tk, :] = sum over
// slices of partial (in slice order) + scale * T[tk].B^T + bias + y_add, one
// grid row (blockIdx.y) per token.  With a LoRA term each CTA first sums the T
// kernel's group partials of its token (all loads in flight, then a
// fixed-order sum per rank) and rounds T[tk] to bf16.  Launched with
// programmatic dependent launch right behind the T kernel (or the GEMM), so
// its launch overlaps their tails; pdl_wait() orders it after both.
constexpr int kFinStage = 8192;  // floats of T partials staged per chunk

__global__ void __launch_bounds__(256)
    gemv_dec_finish_kernel(int M, int N, int slices, GemvEpilogue out) {
  __shared__ float s_t[64];
  extern __shared__ float s_stg[];  // T partials of this token, [t_groups][rank]
  pdl_launch_dependents();
  pdl_wait();
  const int tk = blockIdx.y;
  if (out.rank > 0) {
    const int r = out.rank, G = out.t_groups;
    const int gc = kFinStage / r;  // groups staged per chunk
    const float* src = out.t_part + static_cast<int64_t>(tk) * r;  // [g][M][r]
    float acc = 0.f;                                               // thread j < r: rank j
    for (int g0 = 0; g0 < G; g0 += gc) {
      const int ng = G - g0 < gc ? G - g0 : gc, items = ng * r;
      for (int b = threadIdx.x; b < items; b += 8 * 256) {
        float v[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const int i = b + u * 256;
          v[u] = i < items ? __ldcg(src + static_cast<int64_t>(g0 + i / r) * M * r + i % r) : 0.f;
        }
#pragma unroll
        for (int u = 0; u < 8; ++u)
          if (b + u * 256 < items) s_stg[b + u * 256] = v[u];
      }
      __syncthreads();
      if (threadIdx.x < r)
        for (int g = 0; g < ng; ++g) acc += s_stg[g * r + threadIdx.x];
      __syncthreads();
    }
    if (threadIdx.x < r) {
      const __nv_bfloat16 tb = __float2bfloat16_rn(acc);
      s_t[threadIdx.x] = __bfloat162float(tb);
      if (blockIdx.x == 0 && out.t_dense)
        static_cast<__nv_bfloat16*>(out.t_dense)[static_cast<int64_t>(tk) * r + threadIdx.x] = tb;
    }
    __syncthreads();
  }
  const int64_t total = static_cast<int64_t>(M) * N;
  for (int n = blockIdx.x * blockDim.x + threadIdx.x; n < N; n += gridDim.x * blockDim.x) {
    const int64_t e = static_cast<int64_t>(tk) * N + n;
    float v = 0.f;
    for (int sl = 0; sl < slices; ++sl) v += __ldcg(out.partial + sl * total + e);
    dec_store(out, out.rank > 0 ? s_t : nullptr, N, tk, n, v);
  }
}

// T[tk] of one epilogue into s_t (bf16-rounded, as fp32); all threads of the
// block take part.  Shared by the finishing kernels.
__device__ __forceinline__ void finish_t_row(const GemvEpilogue& out, int M, int tk, float* s_t,
                                             float* s_stg, bool write_dense) {
  const int r = out.rank, G = out.t_groups;
  const int gc = kFinStage / r;
  const float* src = out.t_part + static_cast<int64_t>(tk) * r;
  float acc = 0.f;
  for (int g0 = 0; g0 < G; g0 += gc) {
    const int ng = G - g0 < gc ? G - g0 : gc, items = ng * r;
    for (int b = threadIdx.x; b < items; b += 8 * 256) {
      float v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int i = b + u * 256;
        v[u] = i < items ? __ldcg(src + static_cast<int64_t>(g0 + i / r) * M * r + i % r) : 0.f;
      }
#pragma unroll
      for (int u = 0; u < 8; ++u)
        if (b + u * 256 < items) s_stg[b + u * 256] = v[u];
    }
    __syncthreads();
    if (threadIdx.x < r)
      for (int g = 0; g < ng; ++g) acc += s_stg[g * r + threadIdx.x];
    __syncthreads();
  }
  if (threadIdx.x < r) {
    const __nv_bfloat16 tb = __float2bfloat16_rn(acc);
    s_t[threadIdx.x] = __bfloat162float(tb);
    if (write_dense && out.t_dense)
      static_cast<__nv_bfloat16*>(out.t_dense)[static_cast<int64_t>(tk) * r + threadIdx.x] = tb;
  }
  __syncthreads();
}

// Finishing pass of a grouped launch: the split-K sums and epilogues of up to
// three projections in one grid, blockIdx.x ranges [nb_end[j-1], nb_end[j])
// for projection j.  With act set (two projections of equal N, no LoRA), the
// two results are not stored: act = SwiGLU(first, second) is, with the
// arithmetic of swiglu_fwd_kernel on the bf16-rounded results.
struct GroupFinish {
  GemvEpilogue ep[3];
  int n[3];
  int nb_end[3];
  __nv_bfloat16* act;
};

__global__ void __launch_bounds__(256)
    gemv_group_finish_kernel(int M, int slices, GroupFinish gf) {
  __shared__ float s_t[64];
  extern __shared__ float s_stg[];
  pdl_launch_dependents();
  pdl_wait();
  const int tk = blockIdx.y;
  const int j = blockIdx.x < gf.nb_end[0] ? 0 : blockIdx.x < gf.nb_end[1] ? 1 : 2;
  const int b0 = j == 0 ? 0 : j == 1 ? gf.nb_end[0] : gf.nb_end[1];
  const int nbj = (j == 0 ? gf.nb_end[0] : j == 1 ? gf.nb_end[1] : gf.nb_end[2]) - b0;
  const GemvEpilogue out = j == 0 ? gf.ep[0] : j == 1 ? gf.ep[1] : gf.ep[2];
  const int N = j == 0 ? gf.n[0] : j == 1 ? gf.n[1] : gf.n[2];
  if (out.rank > 0) finish_t_row(out, M, tk, s_t, s_stg, blockIdx.x == b0);
  const int64_t total = static_cast<int64_t>(M) * N;
  for (int n = (blockIdx.x - b0) * blockDim.x + threadIdx.x; n < N; n += nbj * blockDim.x) {
    const int64_t e = static_cast<int64_t>(tk) * N + n;
    float v = 0.f;
    for (int sl = 0; sl < slices; ++sl) v += __ldcg(out.partial + sl * total + e);
    if (gf.act == nullptr) {
      dec_store(out, out.rank > 0 ? s_t : nullptr, N, tk, n, v);
    } else {
      const GemvEpilogue& o2 = gf.ep[1];
      float u = 0.f;
      for (int sl = 0; sl < slices; ++sl) u += __ldcg(o2.partial + sl * total + e);
      const float a = __bfloat162float(__float2bfloat16_rn(dec_value(out, nullptr, N, tk, n, v)));
      const float b = __bfloat162float(__float2bfloat16_rn(dec_value(o2, nullptr, N, tk, n, u)));
      gf.act[e] = __float2bfloat16_rn(swiglu_elem(a, b));
    }
  }
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
        } else if (CH == 1) {
          ck.ca = __ldg(w.absmax_code + ba0 + c0);
          ck.cb = __ldg(w.absmax_code + bb0 + c0);
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
  const int64_t nblk = K / 64;
  const int rts[3] = {16, 8, 4};
  const int kcbs[6] = {128, 64, 32, 16, 8, 4};
  // preferred chunk first; smaller chunks only when no plan fits (few K blocks)
  for (int ch = nt8 <= 2 ? 4 : 2; ch >= 1 && best.rt == 0; ch /= 2) {
    int64_t best_items = -1;
    size_t best_partial = 0;
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
  }
  return best;
}

int ilog2(int v) {
  int l = 0;
  while ((1 << l) < v) ++l;
  return l;
}

// M <= 8 plan: slice = 4*kw blocks dividing K/64; cs = CTAs per slice (at
// most one per tile); the estimate is the tiles of the busiest warp, ties
// broken towards fewer slices (less partial-sum traffic).
Gemv8Plan make_plan8(int64_t m, int64_t N, int64_t K, int num_sms) {
  Gemv8Plan best{};
  const int64_t nblk = K / 64, T = N / 16;
  int64_t best_cost = -1;
  const int qn = m <= 2 ? 1 : m <= 4 ? 2 : 4;
  for (int kw = 16; kw >= 1; kw /= 2) {
    if (nblk % (kw * kDecKB) != 0) continue;
    const int64_t slices = nblk / (kw * kDecKB);
    if (slices > num_sms) continue;
    const int64_t cs = num_sms / slices < T ? num_sms / slices : T;
    const int rtg = kWarps / kw;
    const int64_t per_cta = (T + cs - 1) / cs;
    const int64_t cost = (per_cta + rtg - 1) / rtg;
    if (best_cost < 0 || cost < best_cost) {
      best = Gemv8Plan{kw, rtg, static_cast<int>(cs), static_cast<int>(slices),
                       ilog2(kw), ilog2(rtg), ilog2(qn)};
      best_cost = cost;
    }
  }
  return best;
}

// The M <= 8 kernel when a plan exists (FITQ_GEMV_WIDE=1 forces the general kernel).
bool use_m8(int64_t m, int64_t N, int64_t K, int num_sms, Gemv8Plan* pl) {
  const char* e = getenv("FITQ_GEMV_WIDE");
  if (m > 8 || (e != nullptr && e[0] == '1')) return false;
  *pl = make_plan8(m, N, K, num_sms);
  return pl->kw != 0;
}

}  // namespace

bool gemv_dec_plan(int64_t m, int64_t n_out, int64_t k_in, int num_sms, int* slices) {
  Gemv8Plan pl;
  if (n_out % 16 != 0 || k_in % 256 != 0 || n_out * k_in / 2 >= (1ll << 31)) return false;
  if (!use_m8(m, n_out, k_in, num_sms, &pl)) return false;
  if (slices) *slices = pl.slices;
  return true;
}

bool gemv_dec_needs_partial(int slices, int rank) { return slices > 1 || rank > 0; }

static int launch_dec(const DecJobs& jb, const void* x, int64_t m, const GemvEpilogue& out,
                      const Gemv8Plan& pl, cudaStream_t st);

int launch_nf4_gemv_dec(const Nf4Args& w, const void* x, int64_t m, const GemvEpilogue& out,
                        cudaStream_t st, int num_sms) {
  Gemv8Plan pl;
  if (!gemv_dec_plan(m, w.n_out, w.k_in, num_sms, nullptr) || !use_m8(m, w.n_out, w.k_in, num_sms, &pl))
    return FITQ_ERR_UNSUPPORTED;
  DecJobs jb{};
  jb.w[0] = jb.w[1] = jb.w[2] = w;
  jb.partial[0] = out.partial;
  const int T = static_cast<int>(w.n_out / 16);
  jb.tile0[0] = 0;
  jb.tile0[1] = jb.tile0[2] = jb.tile0[3] = T;
  jb.groups = 1;
  return launch_dec(jb, x, m, out, pl, st);
}

int launch_nf4_gemv_dec_grouped(const Nf4Args* w, int groups, const void* x, int64_t m,
                                float* const* partial, int* status, cudaStream_t st, int num_sms) {
  if (groups < 1 || groups > 3) return FITQ_ERR_UNSUPPORTED;
  int64_t n_total = 0;
  DecJobs jb{};
  jb.tile0[0] = 0;
  for (int g = 0; g < 3; ++g) {
    const int gg = g < groups ? g : groups - 1;
    jb.w[g] = w[gg];
    jb.partial[g] = g < groups ? partial[g] : nullptr;
    if (g < groups) {
      if (w[g].k_in != w[0].k_in || w[g].n_out % 16 != 0 || !partial[g] ||
          (w[g].absmax_f32 == nullptr) != (w[0].absmax_f32 == nullptr))
        return FITQ_ERR_UNSUPPORTED;
      n_total += w[g].n_out;
    }
    jb.tile0[g + 1] = static_cast<int>(n_total / 16);
  }
  jb.groups = groups;
  jb.status = status;
  Gemv8Plan pl;
  if (!gemv_dec_plan(m, n_total, w[0].k_in, num_sms, nullptr) || !use_m8(m, n_total, w[0].k_in, num_sms, &pl))
    return FITQ_ERR_UNSUPPORTED;
  GemvEpilogue out{};  // partials only: the group finishing kernel applies the epilogues
  return launch_dec(jb, x, m, out, pl, st);
}

static int launch_dec(const DecJobs& jb, const void* x, int64_t m, const GemvEpilogue& out,
                      const Gemv8Plan& pl, cudaStream_t st) {
  const Nf4Args& w = jb.w[0];
  auto xb = static_cast<const __nv_bfloat16*>(x);
  const int M = static_cast<int>(m);
  const dim3 grid(static_cast<unsigned>(pl.cs * pl.slices));
  const bool nested = w.absmax_f32 == nullptr;
  if (!set_smem_limit(nested ? nf4_gemv_dec_kernel<true> : nf4_gemv_dec_kernel<false>, kDecSmem))
    return FITQ_ERR_CUDA;
  cudaError_t e =
      nested ? launch_pdl(nf4_gemv_dec_kernel<true>, grid, dim3(kThreads), kDecSmem, st, jb, xb, M, pl, out)
             : launch_pdl(nf4_gemv_dec_kernel<false>, grid, dim3(kThreads), kDecSmem, st, jb, xb, M, pl, out);
  note_launch();
  return e == cudaSuccess ? FITQ_OK : FITQ_ERR_CUDA;
}

// Blocks per token row of the finishing kernels: 128 outputs each (their
// loads of the slice partials and of lora_b are latency-bound, so more blocks
// in flight finish sooner), at most 128.
static int64_t finish_blocks(int64_t n) {
  const int64_t nb = (n + 127) / 128;
  return nb > 128 ? 128 : nb;
}

int launch_nf4_gemv_dec_finish(int64_t m, int64_t n_out, int slices, const GemvEpilogue& out,
                               cudaStream_t st, int num_sms) {
  (void)num_sms;
  if (out.rank > 64) return FITQ_ERR_UNSUPPORTED;
  int64_t nb = finish_blocks(n_out);
  const size_t smem = out.rank > 0 ? kFinStage * sizeof(float) : 0;
  const cudaError_t e = launch_pdl(gemv_dec_finish_kernel,
                                   dim3(static_cast<unsigned>(nb), static_cast<unsigned>(m)), dim3(256),
                                   smem, st, static_cast<int>(m), static_cast<int>(n_out), slices, out);
  note_launch();
  return e == cudaSuccess ? FITQ_OK : FITQ_ERR_CUDA;
}

int launch_nf4_gemv_group_finish(int64_t m, const int64_t* n_out, int jobs, int slices,
                                 const GemvEpilogue* eps, void* swiglu_act, cudaStream_t st) {
  if (jobs < 1 || jobs > 3 || (swiglu_act && (jobs != 2 || n_out[0] != n_out[1]))) return FITQ_ERR_UNSUPPORTED;
  GroupFinish gf{};
  int end = 0, rank_any = 0;
  const int used = swiglu_act ? 1 : jobs;  // SwiGLU: one column range covers both
  for (int j = 0; j < 3; ++j) {
    const int jj = j < jobs ? j : 0;
    gf.ep[j] = eps[jj];
    gf.n[j] = static_cast<int>(n_out[jj]);
    if (eps[jj].rank > 64 || (swiglu_act && eps[jj].rank > 0)) return FITQ_ERR_UNSUPPORTED;
    if (j < used) {
      int64_t nb = finish_blocks(n_out[j]);
      end += static_cast<int>(nb);
      rank_any |= eps[j].rank;
    }
    gf.nb_end[j] = end;
  }
  gf.act = static_cast<__nv_bfloat16*>(swiglu_act);
  const size_t smem = rank_any ? kFinStage * sizeof(float) : 0;
  const cudaError_t e = launch_pdl(gemv_group_finish_kernel,
                                   dim3(static_cast<unsigned>(end), static_cast<unsigned>(m)), dim3(256),
                                   smem, st, static_cast<int>(m), slices, gf);
  note_launch();
  return e == cudaSuccess ? FITQ_OK : FITQ_ERR_CUDA;
}

size_t gemv_partial_bytes(int64_t m, int64_t n_out, int64_t k_in, int num_sms, int* splits_out) {
  const int64_t slices = make_plan(m, n_out, k_in, num_sms).slices;
  if (splits_out) *splits_out = static_cast<int>(slices);
  return static_cast<size_t>(slices * m * n_out) * sizeof(float);
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
  cudaError_t e = cudaSuccess;
#define FITQ_GEMV_CASE(T, C)                                                                      \
  if (p.nt8 == T && p.ch == C) {                                                                  \
    if (!set_smem_limit(nf4_gemv_kernel<T, C>, 200 * 1024)) {                                    \
      e = cudaErrorInvalidValue;                                                                  \
    } else {                                                                                      \
      nf4_gemv_kernel<T, C><<<grid, kThreads, p.smem, st>>>(w, xb, M, p.rt, p.kcb,                \
                                                             static_cast<int>(p.row_groups),      \
                                                             static_cast<int>(items), partial);   \
      note_launch();                                                                              \
    }                                                                                             \
  }
  FITQ_GEMV_CASE(1, 4)
  FITQ_GEMV_CASE(2, 4)
  FITQ_GEMV_CASE(3, 2)
  FITQ_GEMV_CASE(4, 2)
  FITQ_GEMV_CASE(5, 2)
  FITQ_GEMV_CASE(6, 2)
  FITQ_GEMV_CASE(7, 2)
  FITQ_GEMV_CASE(8, 2)
  FITQ_GEMV_CASE(1, 2)
  FITQ_GEMV_CASE(2, 2)
  FITQ_GEMV_CASE(1, 1)
  FITQ_GEMV_CASE(2, 1)
  FITQ_GEMV_CASE(3, 1)
  FITQ_GEMV_CASE(4, 1)
  FITQ_GEMV_CASE(5, 1)
  FITQ_GEMV_CASE(6, 1)
  FITQ_GEMV_CASE(7, 1)
  FITQ_GEMV_CASE(8, 1)
#undef FITQ_GEMV_CASE
  if (e != cudaSuccess) return FITQ_ERR_CUDA;
  *splits_out = static_cast<int>(p.slices);
  return launch_result();
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
  return launch_result();
}

}  // namespace fitq
