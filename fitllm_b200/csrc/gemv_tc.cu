// NF4 skinny GEMM on the 5th-generation tensor cores for the verify and
// small-batch decode row counts (M <= 64):  partial[s][m][n] = x[m, K_s].W[n, K_s]^T
// over K slice s, summed (+ LoRA, bias, residual) by gemv_dec_finish_kernel.
//
// Replaces bitsandbytes matmul_4bit for the speculative-verify shapes
// (fitllm/inference.py:380-397: M = batch x (draft + 1)) and small decode
// batches (fitllm/forward.py:623-625).
//
// The weights are the A operand of tcgen05.mma and live in TENSOR MEMORY:
// one thread per weight row decodes its NF4 bytes (one prmt + one ld.shared
// per byte from a lane-replicated code-pair table, see gemv.cu), scales each
// 64-column block by its absmax (bf16x2 multiply) and writes the bf16 pairs
// into TMEM with tcgen05.st -- exactly A's TMEM layout (row = lane, two
// consecutive K elements per 32-bit column).  The tokens (x, padded to NTOK =
// 16/32/64 rows with zeros) are the B operand, staged in shared memory in the
// 128-byte-swizzled K-major layout.  The tensor core then does all the
// multiply-adds for every token at once, so the decode cost per weight does
// not grow with M.
//
// One CTA per SM, one pipeline (10 warps):
//   warp 0      producer: per stage (two 64-column blocks of one 128-row tile)
//               16-byte cp.async copies of the packed bytes (rows at an 80-byte
//               pitch: conflict-free 16-byte reads; small bulk copies would be
//               issued one request at a time) and of the x tile (zero fill for
//               pad tokens) into an NST-stage ring;
//   warp 1      allocates TMEM (512 columns: four A buffers of 64 columns and
//               the fp32 accumulator) and issues the MMAs from one lane;
//   warps 2-9   decoders: warp w decodes block (w - 2) / 4 of each stage for
//               the 32 rows of TMEM sub-partition w % 4; at the end of an item
//               they drain their half of the accumulator columns and write the
//               fp32 partials.
// Work items are (128-row tile, K slice) pairs, walked by the CTAs with a grid
// stride.  Every mbarrier wait is bounded (common.cuh); no TMA or multicast.
#include "common.cuh"
#include "kernels.cuh"

namespace fitq {
namespace {

constexpr int kTcWarps = 10;
constexpr int kTcThreads = kTcWarps * 32;
constexpr int kTcRows = 128;          // weight rows per tile (UMMA M)
constexpr int kTcWPitch = 80;         // staged bytes per row (64 used)
constexpr int kTcWBytes = kTcRows * kTcWPitch;
constexpr int kTcTbl = 256 * 256;       // code-pair table, 64 KB aligned
constexpr int kTcMaxSt = 8;
constexpr int kTcSmem = 232448 - 2048;  // dynamic shared memory (static part holds barriers)
constexpr int kTcTmemCols = 512;
constexpr int kTcABufs = 4;             // A buffers (64 columns each), then the accumulator
constexpr int kTcAcc = kTcABufs * 64;

struct TcParams {
  Nf4Args w;
  const __nv_bfloat16* x;
  int M;
  int tiles;        // N / 128
  int slices, bps;  // K slices, 64-column blocks per slice (multiple of 4)
  int items;        // tiles * slices
  int nst;          // ring stages
  int stage_bytes;  // x part (2 * NTOK * 128) + W part, multiple of 1024
  float* partial;   // [slices, M, N]
  int* status;
};

extern __shared__ __align__(1024) uint8_t g_tc_smem[];

// 16-byte async copy; src_bytes = 0 fills the destination with zeros.
__device__ __forceinline__ void cp_async16_zfill(uint32_t dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes)
               : "memory");
}

// Arrive on bar once all of this thread's earlier cp.async copies have landed
// (the barrier's expected count includes this arrival).
__device__ __forceinline__ void cp_async_arrive_noinc(uint64_t* bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void umma_bf16_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc,
                                             uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem_d),
      "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate));
}

// 32 lanes x 32 consecutive 32-bit columns: thread i writes lane (base + i).
__device__ __forceinline__ void tmem_st_32x32b_x32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
      "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]),
      "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]),
      "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
__device__ __forceinline__ void tmem_st_wait() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

template <int N>
__device__ __forceinline__ void tmem_ld_32x32b(uint32_t taddr, uint32_t (&r)[N]);
template <>
__device__ __forceinline__ void tmem_ld_32x32b<8>(uint32_t taddr, uint32_t (&r)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]),
                 "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
}
template <>
__device__ __forceinline__ void tmem_ld_32x32b<16>(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, "
      "%12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
template <>
__device__ __forceinline__ void tmem_ld_32x32b<32>(uint32_t taddr, uint32_t (&r)[32]) {
  tmem_ld_32x32b_x32(taddr, r);
}

// bf16 code pair of byte J of v from the 64 KB-aligned table (see gemv.cu).
template <int J>
__device__ __forceinline__ uint32_t tc_tbl(uint32_t v, uint32_t base) {
  uint32_t a, r;
  constexpr uint32_t sel = 0x7600u | (static_cast<uint32_t>(J) << 4) | 4u;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(a) : "r"(v), "r"(base), "n"(sel));
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(r) : "r"(a));
  return r;
}

__device__ __forceinline__ uint32_t hmul2_bf16(uint32_t a, uint32_t b) {
  __nv_bfloat162 r = __hmul2(*reinterpret_cast<const __nv_bfloat162*>(&a),
                             *reinterpret_cast<const __nv_bfloat162*>(&b));
  return *reinterpret_cast<uint32_t*>(&r);
}

// Four bytes of v -> four scaled bf16 pairs.
__device__ __forceinline__ void decode_word(uint32_t v, uint32_t lb, uint32_t am2, uint32_t* o) {
  o[0] = hmul2_bf16(tc_tbl<0>(v, lb), am2);
  o[1] = hmul2_bf16(tc_tbl<1>(v, lb), am2);
  o[2] = hmul2_bf16(tc_tbl<2>(v, lb), am2);
  o[3] = hmul2_bf16(tc_tbl<3>(v, lb), am2);
}

__device__ __forceinline__ uint4 lds128u(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(addr));
  return v;
}

template <int NTOK, bool NESTED>
__global__ void __launch_bounds__(kTcThreads, 1) nf4_gemv_tc_kernel(const TcParams p) {
  __shared__ uint64_t bars[3 * kTcMaxSt + 2 * kTcABufs + 3];
  __shared__ uint32_t tmem_slot;
  __shared__ int abort_s, never_s;
  uint64_t* full = bars;                 // producer -> decoders + MMA (32 cp.async arrivals)
  uint64_t* wfree = bars + kTcMaxSt;     // decoders done with the stage's W (count 8)
  uint64_t* xfree = bars + 2 * kTcMaxSt; // MMAs done with the stage's x (commit)
  uint64_t* afull = bars + 3 * kTcMaxSt; // [kTcABufs] decoders wrote A buffer (count 8)
  uint64_t* aempty = afull + kTcABufs;   // [kTcABufs] MMAs done with A buffer (commit)
  uint64_t* accfull = aempty + kTcABufs; // item's MMAs done (commit)
  uint64_t* accempty = accfull + 1;      // accumulator drained (count 8)
  uint64_t* done = accfull + 2;          // every issued MMA retired (commit)
  volatile int* abort_flag = &abort_s;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int K = static_cast<int>(p.w.k_in), N = static_cast<int>(p.w.n_out);
  const int nblk = K / 64;
  const int nst = p.nst, kst = p.bps / 2;

  // Shared layout: stages in [align1024(base), table) then after the table.
  const uint32_t sbase = smem_u32(g_tc_smem);
  const uint32_t tbl = (sbase + 0xFFFFu) & ~0xFFFFu;
  const uint32_t a0 = (sbase + 1023u) & ~1023u;
  const int n_slack = tbl > a0 ? static_cast<int>((tbl - a0) / p.stage_bytes) : 0;
  const uint32_t after = tbl + kTcTbl;
  auto stage_addr = [&](int s) -> uint32_t {
    return s < n_slack ? a0 + static_cast<uint32_t>(s * p.stage_bytes)
                       : after + static_cast<uint32_t>((s - n_slack) * p.stage_bytes);
  };
  constexpr int kXBytes = 2 * NTOK * 128;  // two 64-column x tiles, 128-byte swizzled

  if (threadIdx.x == 0) {
    for (int s = 0; s < nst; ++s) {
      mbar_init(&full[s], 32);
      mbar_init(&wfree[s], 8);
      mbar_init(&xfree[s], 1);
    }
    for (int a = 0; a < kTcABufs; ++a) {
      mbar_init(&afull[a], 8);
      mbar_init(&aempty[a], 1);
    }
    mbar_init(accfull, 1);
    mbar_init(accempty, 8);
    mbar_init(done, 1);
    abort_s = 0;
    never_s = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(&tmem_slot, kTcTmemCols);
    tmem_relinquish();
  }
  // Everything below reads data written by the predecessor kernel.
  pdl_wait();
  pdl_launch_dependents();
  if (warp >= 2) {
    // entry e (256 B): lanes' bf16 pairs {qm[e >> 4], qm[e & 15]} at 4l, nested map at 128 + 4g
    uint4* table = reinterpret_cast<uint4*>(g_tc_smem + (tbl - sbase));
    for (int i = threadIdx.x - 64; i < 512; i += kTcThreads - 64) {
      const int e = i >> 1, h = i & 1;
      const uint32_t v = pack_bf16x2(__ldg(p.w.quant_map + (e >> 4)), __ldg(p.w.quant_map + (e & 15)));
      const uint4 vv = make_uint4(v, v, v, v);
#pragma unroll
      for (int j = 0; j < 4; ++j) table[e * 16 + h * 4 + j] = vv;
      if (NESTED) {
        const uint32_t nv = __float_as_uint(__ldg(p.w.nested_quant_map + e));
        table[e * 16 + 8 + h] = make_uint4(nv, nv, nv, nv);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = tmem_slot;
  const uint32_t idesc = umma_idesc_bf16_f32(kTcRows, NTOK);

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    int st = 0;
    uint32_t ph = 0;
    bool ok = true;
    for (int it = blockIdx.x; it < p.items && ok; it += gridDim.x) {
      const int t = it / p.slices, sl = it % p.slices;
      const int kb0 = sl * p.bps;
      for (int ks = 0; ks < kst; ++ks) {
        if (!mbar_wait(&wfree[st], ph ^ 1, abort_flag, p.status) ||
            !mbar_wait(&xfree[st], ph ^ 1, abort_flag, p.status)) {
          ok = false;
          break;
        }
        const uint32_t sa = stage_addr(st);
        const int kb = kb0 + 2 * ks;
        // W: 128 rows x 4 chunks of 16 B; chunk c -> row c >> 2, piece c & 3
#pragma unroll 4
        for (int c = lane; c < kTcRows * 4; c += 32) {
          const int r = c >> 2, q = c & 3;
          cp_async16_zfill(sa + kXBytes + r * kTcWPitch + q * 16,
                           p.w.packed + (static_cast<int64_t>(t * kTcRows + r) * nblk + kb) * 32 + q * 16,
                           16u);
        }
        // x tile of each block: NTOK rows x 128 B, chunk q of row tk at q ^ (tk & 7)
        for (int c = lane; c < NTOK * 16; c += 32) {
          const int tk = c >> 4, d = (c >> 3) & 1, q = c & 7;
          const int tks = tk < p.M ? tk : 0;
          const __nv_bfloat16* src = p.x + static_cast<int64_t>(tks) * K + (kb + d) * 64 + q * 8;
          cp_async16_zfill(sa + d * (NTOK * 128) + tk * 128 + ((q ^ (tk & 7)) << 4), src,
                           tk < p.M ? 16u : 0u);
        }
        cp_async_arrive_noinc(&full[st]);
        if (++st == nst) { st = 0; ph ^= 1; }
      }
    }
    asm volatile("cp.async.wait_all;" ::: "memory");
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA
    if (lane == 0) {
      int st = 0, a = 0;
      uint32_t ph = 0, aph = 0, accph = 0;
      bool ok = true;
      const uint32_t acc = tmem_base + kTcAcc;
      for (int it = blockIdx.x; it < p.items && ok; it += gridDim.x) {
        if (!mbar_wait(accempty, accph ^ 1, abort_flag, p.status)) break;
        tc_fence_after();
        for (int ks = 0; ks < kst; ++ks) {
          if (!mbar_wait(&full[st], ph, abort_flag, p.status) ||
              !mbar_wait(&afull[a], aph, abort_flag, p.status)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = stage_addr(st);
#pragma unroll
          for (int d = 0; d < 2; ++d)
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
              umma_bf16_ts(acc, tmem_base + a * 64 + d * 32 + kk * 8,
                           umma_smem_desc_sw128(sa + d * (NTOK * 128) + kk * 32), idesc,
                           (ks > 0 || d > 0 || kk > 0) ? 1u : 0u);
          umma_commit(&aempty[a]);
          umma_commit(&xfree[st]);
          if (++a == kTcABufs) { a = 0; aph ^= 1; }
          if (++st == nst) { st = 0; ph ^= 1; }
        }
        if (!ok) break;
        umma_commit(accfull);
        accph ^= 1;
      }
      // all issued MMAs must retire before TMEM is released
      umma_commit(done);
      mbar_wait(done, 0, &never_s, p.status);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ decoders
    const int d = (warp - 2) >> 2;         // block of the stage this warp decodes
    const int sub = warp & 3;              // TMEM sub-partition (lanes 32 sub .. + 31)
    const int r = sub * 32 + lane;         // row within the tile
    const uint32_t lane_off = static_cast<uint32_t>(sub * 32) << 16;
    const uint32_t lb = tbl | (static_cast<uint32_t>(lane) << 2);
    const uint32_t nq = tbl | (128u + (static_cast<uint32_t>(lane & 7) << 2));
    int st = 0, a = 0;
    uint32_t ph = 0, aph = 0, accph = 0;
    bool ok = true;
    for (int it = blockIdx.x; it < p.items && ok; it += gridDim.x) {
      const int t = it / p.slices, sl = it % p.slices;
      const int row = t * kTcRows + r;
      // Scales, fetched well ahead of use: a 32-bit word of absmax codes covers
      // blocks 4j..4j+3 of the slice, i.e. this thread's blocks of stages 2j and
      // 2j+1 (bytes d and d + 2, one 256-block nested group since 4 | 256); three
      // words (six stages) are in flight.  Plain fp32 absmax: two floats per word.
      const int64_t rb = static_cast<int64_t>(row) * nblk + sl * p.bps;  // 4-aligned (plan)
      const int nwords = p.bps / 4;
      uint32_t c0 = 0, c1 = 0, c2 = 0;
      float n0 = 0.f, n1 = 0.f, n2 = 0.f, m0 = 0.f, m1 = 0.f, m2 = 0.f;
      auto fetch = [&](int j, uint32_t& c, float& n, float& m) {
        if (j >= nwords) return;
        if (NESTED) {
          c = __ldg(reinterpret_cast<const uint32_t*>(p.w.absmax_code + rb) + j);
          n = __ldg(p.w.nested_absmax + ((rb + 4 * j) >> 8));
        } else {
          n = __ldg(p.w.absmax_f32 + rb + 4 * j + d);
          m = __ldg(p.w.absmax_f32 + rb + 4 * j + 2 + d);
        }
      };
      fetch(0, c0, n0, m0);
      fetch(1, c1, n1, m1);
      fetch(2, c2, n2, m2);
      for (int ks = 0; ks < kst; ++ks) {
        const bool odd = ks & 1;
        float am;
        if (NESTED) {
          // code byte d (even stage) or d + 2 (odd stage) of c0 -> nested map entry
          const uint32_t sel = 0x7604u | (static_cast<uint32_t>(d + (odd ? 2 : 0)) << 4);
          uint32_t ca, nv;
          asm("prmt.b32 %0, %1, %2, %3;" : "=r"(ca) : "r"(c0), "r"(nq), "r"(sel));
          asm volatile("ld.shared.u32 %0, [%1];" : "=r"(nv) : "r"(ca));
          am = __fadd_rn(__fmul_rn(__uint_as_float(nv), n0), p.w.offset);
        } else {
          am = odd ? m0 : n0;
        }
        if (odd) {  // word consumed: rotate and fetch three words ahead
          c0 = c1; n0 = n1; m0 = m1;
          c1 = c2; n1 = n2; m1 = m2;
          fetch(ks / 2 + 3, c2, n2, m2);
        }
        const uint32_t am2 = pack_bf16x2(am, am);
        if (!mbar_wait(&full[st], ph, abort_flag, p.status)) { ok = false; break; }
        const uint32_t wrow = stage_addr(st) + kXBytes + r * kTcWPitch + d * 32;
        const uint4 w0 = lds128u(wrow), w1 = lds128u(wrow + 16);
        __syncwarp();
        if (lane == 0) mbar_arrive(&wfree[st]);
        uint32_t o[32];
        decode_word(w0.x, lb, am2, o + 0);
        decode_word(w0.y, lb, am2, o + 4);
        decode_word(w0.z, lb, am2, o + 8);
        decode_word(w0.w, lb, am2, o + 12);
        decode_word(w1.x, lb, am2, o + 16);
        decode_word(w1.y, lb, am2, o + 20);
        decode_word(w1.z, lb, am2, o + 24);
        decode_word(w1.w, lb, am2, o + 28);
        if (!mbar_wait(&aempty[a], aph ^ 1, abort_flag, p.status)) { ok = false; break; }
        tc_fence_after();
        tmem_st_32x32b_x32(tmem_base + lane_off + a * 64 + d * 32, o);
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&afull[a]);
        if (++a == kTcABufs) { a = 0; aph ^= 1; }
        if (++st == nst) { st = 0; ph ^= 1; }
      }
      if (!ok) break;
      // drain this warp's half of the accumulator columns
      if (!mbar_wait(accfull, accph, abort_flag, p.status)) break;
      tc_fence_after();
      uint32_t v[NTOK / 2];
      tmem_ld_32x32b<NTOK / 2>(tmem_base + lane_off + kTcAcc + d * (NTOK / 2), v);
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(accempty);
      accph ^= 1;
      float* out = p.partial + static_cast<int64_t>(sl) * p.M * N + row;
#pragma unroll
      for (int j = 0; j < NTOK / 2; ++j) {
        const int tk = d * (NTOK / 2) + j;
        if (tk < p.M) out[static_cast<int64_t>(tk) * N] = __uint_as_float(v[j]);
      }
    }
  }

  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTcTmemCols);
  }
}

struct TcPlan {
  int ntok, slices, bps, items, grid, nst, stage_bytes;
};

// Slices (block counts that are multiples of 4 dividing K/64) minimising the busiest CTA's weight
// bytes plus the split-K partial traffic, over `sms` CTAs.
TcPlan make_tc_plan(int64_t m, int64_t N, int64_t K, int sms) {
  TcPlan best{};
  const int64_t nblk = K / 64, tiles = N / kTcRows;
  const int ntok = m <= 16 ? 16 : m <= 32 ? 32 : 64;
  const int stage_bytes = 2 * ntok * 128 + ((kTcWBytes + 1023) / 1024) * 1024;
  int nst = (kTcSmem - 1024 - stage_bytes - kTcTbl) / stage_bytes;
  if (nst > kTcMaxSt) nst = kTcMaxSt;
  double best_cost = -1.0;
  for (int64_t bps = 4; bps <= nblk; bps += 4) {
    if (nblk % bps != 0) continue;
    const int64_t slices = nblk / bps;
    const int64_t items = tiles * slices;
    const int64_t grid = items < sms ? items : sms;
    const int64_t per_cta = (items + grid - 1) / grid;
    const double wbytes = static_cast<double>(per_cta) * bps * kTcRows * 32.0 * sms;  // busiest CTA x sms
    const double pbytes = 2.0 * slices * m * N * 4.0;
    const double cost = wbytes + pbytes;
    if (best_cost < 0 || cost < best_cost) {
      best = TcPlan{ntok, static_cast<int>(slices), static_cast<int>(bps), static_cast<int>(items),
                    static_cast<int>(grid), nst, stage_bytes};
      best_cost = cost;
    }
  }
  return best;
}

}  // namespace

bool gemv_tc_plan(int64_t m, int64_t n_out, int64_t k_in, int num_sms, int* slices) {
  const char* e = getenv("FITQ_GEMV_TC");
  const int64_t lo = (e != nullptr && e[0] == '1') ? 1 : 9;  // FITQ_GEMV_TC=1: also M <= 8
  if (e != nullptr && e[0] == '0') return false;
  if (m < lo || m > 64 || n_out % kTcRows != 0 || k_in % 256 != 0) return false;
  if (n_out * k_in / 2 >= (1ll << 31)) return false;
  const TcPlan pl = make_tc_plan(m, n_out, k_in, num_sms);
  if (pl.slices == 0 || pl.nst < 2) return false;
  if (slices) *slices = pl.slices;
  return true;
}

int launch_nf4_gemv_tc(const Nf4Args& w, const void* x, int64_t m, float* partial, int* status,
                       cudaStream_t st, int num_sms) {
  const TcPlan pl = make_tc_plan(m, w.n_out, w.k_in, num_sms);
  if (pl.slices == 0 || pl.nst < 2) return FITQ_ERR_UNSUPPORTED;
  if ((reinterpret_cast<uintptr_t>(w.absmax_code) & 3) != 0) return FITQ_ERR_ALIGN;  // word reads
  TcParams p;
  p.w = w;
  p.x = static_cast<const __nv_bfloat16*>(x);
  p.M = static_cast<int>(m);
  p.tiles = static_cast<int>(w.n_out / kTcRows);
  p.slices = pl.slices;
  p.bps = pl.bps;
  p.items = pl.items;
  p.nst = pl.nst;
  p.stage_bytes = pl.stage_bytes;
  p.partial = partial;
  p.status = status;
  const bool nested = w.absmax_f32 == nullptr;
  cudaError_t e = cudaSuccess;
#define FITQ_TC_CASE(NT)                                                                        \
  if (pl.ntok == NT) {                                                                          \
    static bool attr[2] = {false, false};                                                       \
    auto kern = nested ? nf4_gemv_tc_kernel<NT, true> : nf4_gemv_tc_kernel<NT, false>;          \
    if (!attr[nested]) {                                                                        \
      e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kTcSmem);     \
      if (e != cudaSuccess) return FITQ_ERR_CUDA;                                               \
      attr[nested] = true;                                                                      \
    }                                                                                           \
    e = launch_pdl(kern, dim3(static_cast<unsigned>(pl.grid)), dim3(kTcThreads), kTcSmem, st, p); \
  }
  FITQ_TC_CASE(16)
  FITQ_TC_CASE(32)
  FITQ_TC_CASE(64)
#undef FITQ_TC_CASE
  note_launch();
  return e == cudaSuccess ? FITQ_OK : FITQ_ERR_CUDA;
}

}  // namespace fitq
