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
// 16/32/48/64 rows with zeros) are the B operand, staged in shared memory in
// the 128-byte-swizzled K-major layout.  The tensor core then does all the
// multiply-adds for every token at once, so the decode cost per weight does
// not grow with M.
//
// A stage is four 64-column blocks (256 K values) of one 128-row tile: its
// packed bytes (16 KB) and the four matching x tiles.  One CTA per SM, 21 warps:
//   warp 0      producer: per stage one TMA load of the packed bytes (128 rows
//               x 128 B, 128-byte swizzle: conflict-free 16-byte reads by row)
//               and four of the x tiles (tokens >= M read as zeros), issued
//               together on one barrier.  Loads leave the TMA unit in order,
//               so x issued later than its weights would wait behind every
//               weight load queued in between;
//   warps 1-4   MMA issuers: one lane of warp 1 + b issues the four MMAs of
//               block b of every stage into its own fp32 accumulator.  One
//               thread waits about 50 cycles on each M=128, K=16 MMA whatever
//               N <= 64 is; four issuers (one per SM sub-partition) bring a
//               stage's 16 MMAs to the tensor core's own rate.  Warp 1 also
//               allocates TMEM: A buffers of 128 columns (three for NTOK <= 32,
//               two above) and the four accumulators;
//   warps 5-20  decoders: warp w decodes block (w - 5) / 4 of every stage for
//               the 32 rows of TMEM sub-partition w % 4; at the end of an item
//               each drains NTOK / 4 columns of the four accumulators and
//               writes their sum as the fp32 partials.
// Work items are (128-row tile, K slice) pairs, walked by the CTAs with a grid
// stride.  One launch may cover up to three weights that share K and x (q, k
// and v, or gate and up): the tiles of all of them form one item list, each
// with its own tensor map, scales and partial-sum buffer, so small weights
// (k, v: 8 tiles each) share the SMs instead of each splitting K many ways.  Every mbarrier wait is bounded (common.cuh); no multicast.
#include "common.cuh"
#include "kernels.cuh"

namespace fitq {
namespace {

constexpr int kTcWarps = 21;
constexpr int kTcThreads = kTcWarps * 32;
constexpr int kTcDecWarp0 = 5;          // first decoder warp (issuers are warps 1-4)
constexpr int kTcRows = 128;            // weight rows per tile (UMMA M)
constexpr int kTcWStage = kTcRows * 128;  // packed bytes of one stage (four blocks per row)
constexpr int kTcTbl = 256 * 256;       // code-pair table, 64 KB aligned
constexpr int kTcMaxSt = 8;
constexpr int kTcSmem = 232448 - 2048;  // dynamic shared memory (static part holds barriers)
constexpr int kTcTmemCols = 512;
constexpr int kTcMaxABufs = 3;          // A buffers (128 columns each), then the accumulators
// TMEM plan per token padding: A buffers, first accumulator column, column
// stride of the four accumulators (3 x 128 + 4 x 32 or 2 x 128 + 4 x 64 = 512).
__host__ __device__ constexpr int tc_abufs(int ntok) { return ntok <= 32 ? 3 : 2; }
__host__ __device__ constexpr int tc_acc_stride(int ntok) { return ntok <= 32 ? 32 : 64; }

constexpr int kTcMaxGroups = 3;

struct TcParams {
  Nf4Args w[kTcMaxGroups];          // weights of the launch (same K, same scale format)
  float* partial[kTcMaxGroups];     // [slices, M, N_g] each
  int tile_end[kTcMaxGroups];       // exclusive prefix sums of the groups' tiles
  int groups;
  int M;
  int tiles;        // total tiles of all groups
  int slices, bps;  // K slices, 64-column blocks per slice (multiple of 4)
  int items;        // tiles * slices
  int nst;          // ring stages
  int xbytes;       // x bytes of one stage (4 * NTOK * 128)
  int* status;
};

// Group of a (global) tile index and its first tile.
__device__ __forceinline__ int tc_group(const TcParams& p, int t) {
  return t < p.tile_end[0] ? 0 : t < p.tile_end[1] ? 1 : 2;
}
__device__ __forceinline__ int tc_group_start(const TcParams& p, int g) {
  return g == 0 ? 0 : g == 1 ? p.tile_end[0] : p.tile_end[1];
}

extern __shared__ __align__(1024) uint8_t g_tc_smem[];

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

// 32 lanes x 4 consecutive 32-bit columns: thread i reads lane (base + i).
__device__ __forceinline__ void tmem_ld_32x32b_x4(uint32_t taddr, uint32_t (&r)[4]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(taddr));
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
__global__ void __launch_bounds__(kTcThreads, 1)
    nf4_gemv_tc_kernel(const __grid_constant__ CUtensorMap tm_w0,
                       const __grid_constant__ CUtensorMap tm_w1,
                       const __grid_constant__ CUtensorMap tm_w2,
                       const __grid_constant__ CUtensorMap tm_x, const TcParams p) {
  __shared__ uint64_t bars[3 * kTcMaxSt + 2 * kTcMaxABufs + 3];
  __shared__ uint32_t slot_s[2 * kTcMaxSt];  // W slot of stage s at [s], x slot at [kTcMaxSt + s]
  __shared__ uint32_t tmem_slot;
  __shared__ int abort_s, never_s, layout_ok_s;
  uint64_t* full = bars;                  // producer -> decoders + MMA (TMA bytes, W and x)
  uint64_t* wfree = full + kTcMaxSt;      // decoders read the W slot (count 16)
  constexpr int kABufs = tc_abufs(NTOK), kAccStride = tc_acc_stride(NTOK);
  constexpr int kAcc = kABufs * 128;      // accumulator of issuer b at kAcc + b kAccStride
  uint64_t* xfree = wfree + kTcMaxSt;     // MMAs done with the x slot (4 commits)
  uint64_t* afull = xfree + kTcMaxSt;     // [kABufs] decoders wrote A buffer (count 16)
  uint64_t* aempty = afull + kTcMaxABufs; // [kABufs] MMAs done with A buffer (4 commits)
  uint64_t* accfull = aempty + kTcMaxABufs;  // item's MMAs done (4 commits)
  uint64_t* accempty = accfull + 1;       // accumulators drained (count 16)
  uint64_t* done = accfull + 2;           // every issued MMA retired (4 commits)
  volatile int* abort_flag = &abort_s;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int K = static_cast<int>(p.w[0].k_in);
  const int nblk = K / 64;
  const int nst = p.nst, kst = p.bps / 4;

  // Shared layout: the 64 KB-aligned table, ring slots first-fit before and after it.
  const uint32_t sbase = smem_u32(g_tc_smem);
  const uint32_t tbl = (sbase + 0xFFFFu) & ~0xFFFFu;
  if (threadIdx.x == 0) {
    uint32_t cur_a = (sbase + 1023u) & ~1023u, cur_b = tbl + kTcTbl;
    const uint32_t end = sbase + kTcSmem;
    bool ok = nst <= kTcMaxSt;
    auto place = [&](int i, uint32_t bytes) {
      if (cur_a + bytes <= tbl) { slot_s[i] = cur_a; cur_a += bytes; }
      else { slot_s[i] = cur_b; cur_b += bytes; }
    };
    for (int i = 0; ok && i < nst; ++i) place(kTcMaxSt + i, static_cast<uint32_t>(p.xbytes));
    for (int i = 0; ok && i < nst; ++i) place(i, kTcWStage);
    if (cur_b > end) ok = false;
    layout_ok_s = ok ? 1 : 0;
    if (!ok) report_device_error(p.status, FITQ_ERR_UNSUPPORTED);
    for (int s = 0; s < kTcMaxSt; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&wfree[s], 16);
      mbar_init(&xfree[s], 4);
    }
    for (int a = 0; a < kABufs; ++a) {
      mbar_init(&afull[a], 16);
      mbar_init(&aempty[a], 4);
    }
    mbar_init(accfull, 4);
    mbar_init(accempty, 16);
    mbar_init(done, 4);
    abort_s = 0;
    never_s = 0;
    fence_mbar_init();
  }
  __syncthreads();
  if (!layout_ok_s) return;
  if (warp == 1) {
    tmem_alloc(&tmem_slot, kTcTmemCols);
    tmem_relinquish();
  }
  // Everything below reads data written by the predecessor kernel.
  pdl_wait();
  pdl_launch_dependents();
  if (warp >= kTcDecWarp0) {
    // entry e (256 B): lanes' bf16 pairs {qm[e >> 4], qm[e & 15]} at 4l, nested map at 128 + 4g
    uint4* table = reinterpret_cast<uint4*>(g_tc_smem + (tbl - sbase));
    constexpr int kFill = kTcThreads - 32 * kTcDecWarp0;
    for (int i = threadIdx.x - 32 * kTcDecWarp0; i < 512; i += kFill) {
      const int e = i >> 1, h = i & 1;
      const float qa = __ldg(p.w[0].quant_map + (e >> 4)), qb = __ldg(p.w[0].quant_map + (e & 15));
      const uint32_t v = pack_bf16x2(qa, qb);
      const uint4 vv = make_uint4(v, v, v, v);
#pragma unroll
      for (int j = 0; j < 4; ++j) table[e * 16 + h * 4 + j] = vv;
      if (NESTED) {
        const uint32_t nv = __float_as_uint(__ldg(p.w[0].nested_quant_map + e));
        table[e * 16 + 8 + h] = make_uint4(nv, nv, nv, nv);
      }
    }
    // One code table serves every group: the groups' maps must hold the same values.
    const int i = threadIdx.x - 32 * kTcDecWarp0;
    for (int g = 1; g < p.groups; ++g) {
      bool same = true;
      if (i < 16) same = __ldg(p.w[g].quant_map + i) == __ldg(p.w[0].quant_map + i);
      if (NESTED && i < 256)
        same = same && __ldg(p.w[g].nested_quant_map + i) == __ldg(p.w[0].nested_quant_map + i);
      if (!same) report_device_error(p.status, FITQ_ERR_UNSUPPORTED);
    }
  }
  // The producer needs neither the table nor TMEM: it starts streaming now and
  // the other warps wait for both on a named barrier of their own.
  if (warp != 0) {
    tc_fence_before();
    asm volatile("bar.sync 1, %0;" ::"n"(kTcThreads - 32) : "memory");
    tc_fence_after();
  }
  const uint32_t tmem_base = tmem_slot;
  const uint32_t idesc = umma_idesc_bf16_f32(kTcRows, NTOK);
  constexpr int kXTile = NTOK * 128;  // one 64-column x tile, 128-byte swizzled

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      tma_prefetch_desc(&tm_w0);
      if (p.groups > 1) tma_prefetch_desc(&tm_w1);
      if (p.groups > 2) tma_prefetch_desc(&tm_w2);
      tma_prefetch_desc(&tm_x);
      int st = 0;
      uint32_t ph = 0;
      uint32_t armed = 0, armed_parity = 0;  // per-stage bit: armed / parity of the last arm
      bool ok = true;
      for (int it = blockIdx.x; it < p.items && ok; it += gridDim.x) {
        const int tg = it / p.slices, sl = it % p.slices;
        const int g = tc_group(p, tg), t = tg - tc_group_start(p, g);
        const CUtensorMap* tm_w = g == 0 ? &tm_w0 : g == 1 ? &tm_w1 : &tm_w2;
        const int kb0 = sl * p.bps;
        for (int ks = 0; ks < kst; ++ks) {
          if (!mbar_wait(&wfree[st], ph ^ 1, abort_flag, p.status) ||
              !mbar_wait(&xfree[st], ph ^ 1, abort_flag, p.status)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[st], kTcWStage + p.xbytes);
          armed |= 1u << st;
          armed_parity = (armed_parity & ~(1u << st)) | (ph << st);
          const int kb = kb0 + 4 * ks;
          // packed bytes: x = byte column kb * 32 (a multiple of 128), y = first row of the tile
          tma_load_2d(g_tc_smem + (slot_s[st] - sbase), tm_w, &full[st], kb * 32, t * kTcRows);
          uint8_t* xd = g_tc_smem + (slot_s[kTcMaxSt + st] - sbase);
#pragma unroll
          for (int b = 0; b < 4; ++b) tma_load_2d(xd + b * kXTile, &tm_x, &full[st], (kb + b) * 64, 0);
          if (++st == nst) { st = 0; ph ^= 1; }
        }
      }
      // Never leave a bulk copy in flight: wait for the last arm of each stage.
      for (int s = 0; s < nst; ++s)
        if (armed & (1u << s)) mbar_wait(&full[s], (armed_parity >> s) & 1u, &never_s, p.status);
    }
    __syncwarp();
  } else if (warp < kTcDecWarp0) {
    // ------------------------------------------------------------ MMA issuers
    if (lane == 0) {
      const int blk = warp - 1;  // block of every stage this thread multiplies
      int xs = 0, a = 0;
      uint32_t xph = 0, aph = 0, accph = 0;  // x slot = ring stage
      bool ok = true;
      const uint32_t acc = tmem_base + kAcc + kAccStride * blk;
      for (int it = blockIdx.x; it < p.items && ok; it += gridDim.x) {
        if (!mbar_wait(accempty, accph ^ 1, abort_flag, p.status)) break;
        tc_fence_after();
        for (int ks = 0; ks < kst; ++ks) {
          if (!mbar_wait(&full[xs], xph, abort_flag, p.status) ||
              !mbar_wait(&afull[a], aph, abort_flag, p.status)) {
            ok = false;
            break;
          }
          tc_fence_after();
          // Keep the per-MMA work to two adds: both offsets stay inside the
          // 14-bit start-address field (shared addresses < 256 KB).
          const uint64_t xd = umma_smem_desc_sw128(slot_s[kTcMaxSt + xs] + blk * kXTile);
          const uint32_t ad = tmem_base + a * 128 + 32 * blk;
          umma_bf16_ts(acc, ad, xd, idesc, ks > 0 ? 1u : 0u);
#pragma unroll
          for (int kk = 1; kk < 4; ++kk)
            umma_bf16_ts(acc, ad + kk * 8, xd + static_cast<uint64_t>((kk * 32) >> 4), idesc, 1u);
          umma_commit(&aempty[a]);
          umma_commit(&xfree[xs]);
          if (++a == kABufs) { a = 0; aph ^= 1; }
          if (++xs == nst) { xs = 0; xph ^= 1; }
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
    const int d = (warp - kTcDecWarp0) >> 2;  // block of the stage this warp decodes
    const int sub = warp & 3;                 // TMEM sub-partition (lanes 32 sub .. + 31)
    const int r = sub * 32 + lane;            // row within the tile
    const uint32_t lane_off = static_cast<uint32_t>(sub * 32) << 16;
    const uint32_t lb = tbl | (static_cast<uint32_t>(lane) << 2);
    const uint32_t nq = tbl | (128u + (static_cast<uint32_t>(lane & 7) << 2));
    const uint32_t csel = 0x7604u | (static_cast<uint32_t>(d) << 4);  // absmax code byte d
    // 128-byte swizzle: 16-byte chunk c of row r sits at chunk c ^ (r & 7)
    const uint32_t w_off0 = static_cast<uint32_t>(r * 128) + (((2u * d) ^ (r & 7u)) << 4);
    const uint32_t w_off1 = static_cast<uint32_t>(r * 128) + (((2u * d + 1u) ^ (r & 7u)) << 4);
    int ws = 0, a = 0;
    uint32_t wph = 0, aph = 0, accph = 0;
    bool ok = true;
    for (int it = blockIdx.x; it < p.items && ok; it += gridDim.x) {
      const int tg = it / p.slices, sl = it % p.slices;
      const int g = tc_group(p, tg), t = tg - tc_group_start(p, g);
      const int row = t * kTcRows + r;
      const int N = static_cast<int>(g == 0 ? p.w[0].n_out : g == 1 ? p.w[1].n_out : p.w[2].n_out);
      const uint8_t* acode = g == 0 ? p.w[0].absmax_code : g == 1 ? p.w[1].absmax_code : p.w[2].absmax_code;
      const float* nabs = g == 0 ? p.w[0].nested_absmax : g == 1 ? p.w[1].nested_absmax : p.w[2].nested_absmax;
      const float* af32 = g == 0 ? p.w[0].absmax_f32 : g == 1 ? p.w[1].absmax_f32 : p.w[2].absmax_f32;
      const float offset = g == 0 ? p.w[0].offset : g == 1 ? p.w[1].offset : p.w[2].offset;
      float* const part = g == 0 ? p.partial[0] : g == 1 ? p.partial[1] : p.partial[2];
      // Scales, fetched three stages ahead: the 32-bit word j of absmax codes
      // covers blocks 4j..4j+3 of the slice (stage j; one 256-block nested
      // group since 4 | 256), this warp's block is byte d.
      const int64_t rb = static_cast<int64_t>(row) * nblk + sl * p.bps;  // 4-aligned (plan)
      uint32_t c0 = 0, c1 = 0, c2 = 0;
      float n0 = 0.f, n1 = 0.f, n2 = 0.f;
      auto fetch = [&](int j, uint32_t& c, float& n) {
        if (j >= kst) return;
        if (NESTED) {
          c = __ldg(reinterpret_cast<const uint32_t*>(acode + rb) + j);
          n = __ldg(nabs + ((rb + 4 * j) >> 8));
        } else {
          n = __ldg(af32 + rb + 4 * j + d);
        }
      };
      fetch(0, c0, n0);
      fetch(1, c1, n1);
      fetch(2, c2, n2);
      for (int ks = 0; ks < kst; ++ks) {
        float am;
        if (NESTED) {
          uint32_t ca, nv;
          asm("prmt.b32 %0, %1, %2, %3;" : "=r"(ca) : "r"(c0), "r"(nq), "r"(csel));
          asm volatile("ld.shared.u32 %0, [%1];" : "=r"(nv) : "r"(ca));
          am = __fadd_rn(__fmul_rn(__uint_as_float(nv), n0), offset);
        } else {
          am = n0;
        }
        c0 = c1; n0 = n1;
        c1 = c2; n1 = n2;
        fetch(ks + 3, c2, n2);
        const uint32_t am2 = pack_bf16x2(am, am);
        if (!mbar_wait(&full[ws], wph, abort_flag, p.status)) { ok = false; break; }
        const uint32_t wa = slot_s[ws];
        const uint4 w0 = lds128u(wa + w_off0);
        const uint4 w1 = lds128u(wa + w_off1);
        __syncwarp();
        if (lane == 0) mbar_arrive(&wfree[ws]);
        if (++ws == nst) { ws = 0; wph ^= 1; }
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
        tmem_st_32x32b_x32(tmem_base + lane_off + a * 128 + d * 32, o);
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&afull[a]);
        if (++a == kABufs) { a = 0; aph ^= 1; }
      }
      if (!ok) break;
      // drain this warp's quarter of the columns of the four accumulators
      if (!mbar_wait(accfull, accph, abort_flag, p.status)) break;
      tc_fence_after();
      constexpr int kQ = NTOK / 4;
      float v[kQ];
#pragma unroll
      for (int q = 0; q < kQ; q += 4) {
        uint32_t v0[4], v1[4], v2[4], v3[4];
        const uint32_t col = tmem_base + lane_off + kAcc + d * kQ + q;
        tmem_ld_32x32b_x4(col, v0);
        tmem_ld_32x32b_x4(col + kAccStride, v1);
        tmem_ld_32x32b_x4(col + 2 * kAccStride, v2);
        tmem_ld_32x32b_x4(col + 3 * kAccStride, v3);
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 4; ++j)
          v[q + j] = (__uint_as_float(v0[j]) + __uint_as_float(v1[j])) +
                     (__uint_as_float(v2[j]) + __uint_as_float(v3[j]));
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(accempty);
      accph ^= 1;
      float* out = part + static_cast<int64_t>(sl) * p.M * N + row;
#pragma unroll
      for (int j = 0; j < kQ; ++j) {
        const int tk = d * kQ + j;
        if (tk < p.M) out[static_cast<int64_t>(tk) * N] = v[j];
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
  int ntok, slices, bps, items, grid, nst, xbytes;
};

// Token padding, ring depth and the K slicing (block counts that are multiples
// of 4 dividing K/64) minimising the busiest CTA's weight bytes plus the
// split-K partial traffic, over `sms` CTAs.  Ring depths are those whose slots
// fit by first-fit around the 64 KB-aligned table for any static shared size
// up to 2 KB.
TcPlan make_tc_plan(int64_t m, int64_t N, int64_t K, int sms) {
  TcPlan best{};
  const int64_t nblk = K / 64, tiles = N / kTcRows;
  const int ntok = m <= 16 ? 16 : m <= 32 ? 32 : m <= 48 ? 48 : 64;
  const int xbytes = 4 * ntok * 128;
  const int nst = ntok == 16 ? 6 : ntok == 32 ? 4 : 3;
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
                    static_cast<int>(grid), nst, xbytes};
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
  if (pl.slices == 0) return false;
  if (slices) *slices = pl.slices;
  return true;
}

int launch_nf4_gemv_tc_grouped(const Nf4Args* w, int groups, const void* x, int64_t m,
                               float* const* partial, int* status, cudaStream_t st, int num_sms) {
  if (groups < 1 || groups > kTcMaxGroups) return FITQ_ERR_UNSUPPORTED;
  const bool nested = w[0].absmax_f32 == nullptr;
  int64_t n_total = 0;
  for (int g = 0; g < groups; ++g) {
    if (w[g].k_in != w[0].k_in || w[g].n_out % kTcRows != 0 || (w[g].absmax_f32 == nullptr) != nested)
      return FITQ_ERR_UNSUPPORTED;
    if (nested && (reinterpret_cast<uintptr_t>(w[g].absmax_code) & 3) != 0) return FITQ_ERR_ALIGN;
    if ((reinterpret_cast<uintptr_t>(w[g].packed) & 15) != 0) return FITQ_ERR_ALIGN;  // TMA source
    n_total += w[g].n_out;
  }
  if ((reinterpret_cast<uintptr_t>(x) & 15) != 0) return FITQ_ERR_ALIGN;  // TMA source
  const int64_t K = w[0].k_in;
  const TcPlan pl = make_tc_plan(m, n_total, K, num_sms);
  if (pl.slices == 0) return FITQ_ERR_UNSUPPORTED;
  CUtensorMap tm_w[kTcMaxGroups], tm_x;
  for (int g = 0; g < groups; ++g)
    if (!encode_tmap_2d(&tm_w[g], CU_TENSOR_MAP_DATA_TYPE_UINT8, w[g].packed, K / 2, w[g].n_out, K / 2,
                        128u, kTcRows, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B))
      return FITQ_ERR_CUDA;
  for (int g = groups; g < kTcMaxGroups; ++g) tm_w[g] = tm_w[0];
  if (!encode_tmap_2d(&tm_x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, x, K, m, K * 2, 64u,
                      static_cast<uint32_t>(pl.ntok), CU_TENSOR_MAP_SWIZZLE_128B,
                      CU_TENSOR_MAP_L2_PROMOTION_L2_128B))
    return FITQ_ERR_CUDA;
  TcParams p;
  int end = 0;
  for (int g = 0; g < kTcMaxGroups; ++g) {
    const int gg = g < groups ? g : 0;
    p.w[g] = w[gg];
    p.partial[g] = partial[gg];
    if (g < groups) end += static_cast<int>(w[g].n_out / kTcRows);
    p.tile_end[g] = end;
  }
  p.groups = groups;
  p.M = static_cast<int>(m);
  p.tiles = end;
  p.slices = pl.slices;
  p.bps = pl.bps;
  p.items = pl.items;
  p.nst = pl.nst;
  p.xbytes = pl.xbytes;
  p.status = status;
  cudaError_t e = cudaSuccess;
#define FITQ_TC_CASE(NT)                                                                        \
  if (pl.ntok == NT) {                                                                          \
    auto kern = nested ? nf4_gemv_tc_kernel<NT, true> : nf4_gemv_tc_kernel<NT, false>;          \
    if (!set_smem_limit(kern, kTcSmem)) return FITQ_ERR_CUDA;                                   \
    e = launch_pdl(kern, dim3(static_cast<unsigned>(pl.grid)), dim3(kTcThreads), kTcSmem, st,     \
                   tm_w[0], tm_w[1], tm_w[2], tm_x, p);                                         \
  }
  FITQ_TC_CASE(16)
  FITQ_TC_CASE(32)
  FITQ_TC_CASE(48)
  FITQ_TC_CASE(64)
#undef FITQ_TC_CASE
  note_launch();
  return e == cudaSuccess ? FITQ_OK : FITQ_ERR_CUDA;
}

int launch_nf4_gemv_tc(const Nf4Args& w, const void* x, int64_t m, float* partial, int* status,
                       cudaStream_t st, int num_sms) {
  return launch_nf4_gemv_tc_grouped(&w, 1, x, m, &partial, status, st, num_sms);
}

}  // namespace fitq
