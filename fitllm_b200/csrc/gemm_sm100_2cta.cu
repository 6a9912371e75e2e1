// tcgen05 GEMM on CTA pairs (cta_group::2): C = A.B^T (+ LoRA K-block)
// (+ bias) (+ C_add), 256 x 256 output tile per pair.
//
// A cluster of two CTAs on neighbouring SMs shares one MMA: CTA r holds rows
// [128r, 128r+128) of the A tile and rows [128r, 128r+128) of the B tile in
// its own shared memory (each CTA TMA-loads only its own halves -- no
// multicast); the leader CTA (rank 0) issues tcgen05.mma.cta_group::2 with
// M = 256, N = 256, which reads both CTAs' shared memory and accumulates rows
// [128r, 128r+128) x 256 columns into CTA r's TMEM.  Per SM this halves the
// B-operand shared-memory / L2 traffic of the one-CTA 128x256 tile.
//
// Synchronisation: both CTAs' TMA loads complete on the leader's "full"
// barrier (armed by the leader with the pair's byte count); the leader's
// commits are multicast to both CTAs' "empty" (stage free) and "tfull"
// (accumulator ready) barriers; both CTAs' epilogue warps arrive on the
// leader's "tempty" barrier.  Every wait is bounded (common.cuh).
#include <cstdlib>

#include "common.cuh"
#include "kernels.cuh"
#include "pair.cuh"

namespace fitq {
namespace {

// Output columns per pair tile, BN, is a template parameter (a multiple of
// 16; each CTA loads BN / 2 rows of B): 256 by default, narrower when the
// 256-wide grid would leave most pairs idle (few rows).  The two
// accumulators sit 256 TMEM columns apart whatever BN is.
constexpr int BM = 128;        // rows of A per CTA (pair tile: 256)
constexpr int BK = 64;
constexpr int STAGES = 6;
constexpr int A_BYTES = BM * BK * 2;
constexpr int NUM_THREADS = 192;
constexpr int NUM_ACC = 2;
constexpr int ACC_STRIDE = 256;
constexpr int TMEM_COLS = 512;
constexpr int GROUP_M = 8;  // in pair tiles (256 rows)
template <int BN>
struct PairTile {
  static constexpr int BN_HALF = BN / 2;                 // rows of B per CTA
  static constexpr int B_BYTES = BN_HALF * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr size_t SMEM_BYTES = 1024 + STAGES * STAGE_BYTES + 256;
};

struct Params {
  __nv_bfloat16* c;
  const __nv_bfloat16* c_add;
  const __nv_bfloat16* bias;
  int64_t ldc, ldc_add;
  int m, n, k;
  int lora_k;
  int num_m, num_n;
  int group_m;  // M-tiles per raster group (L2 reuse of the B tiles)  // in pair tiles
  int* status;
  int epi;                        // GEMM_EPI_* (kernels.cuh)
  const __nv_bfloat16* src0;      // DSWIGLU: gate [m, n]
  const __nv_bfloat16* src1;      // DSWIGLU: up [m, n]
  __nv_bfloat16* aux0;            // SWIGLU: gate out; DSWIGLU: d_up
  __nv_bfloat16* aux1;            // SWIGLU: up out
};

__device__ __forceinline__ void tile_coords(int tile, int num_m, int num_n, int group_m, int& mb,
                                            int& nb) {
  const int per_group = group_m * num_n;
  const int group = tile / per_group;
  const int first_m = group * group_m;
  const int gsz = min(num_m - first_m, group_m);
  const int local = tile - group * per_group;
  mb = first_m + local % gsz;
  nb = local / gsz;
}

__device__ __forceinline__ void add_bf16x8(float (&f)[8], const __nv_bfloat16* p) {
  const uint4 q = *reinterpret_cast<const uint4*>(p);
  const uint32_t qa[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float2 t = unpack_bf16x2(qa[j]);
    f[2 * j] += t.x;
    f[2 * j + 1] += t.y;
  }
}

template <int BN>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(NUM_THREADS, 1)
    gemm_bf16_tn_2cta_kernel(const __grid_constant__ CUtensorMap tm_a,
                             const __grid_constant__ CUtensorMap tm_b,
                             const __grid_constant__ CUtensorMap tm_pa,
                             const __grid_constant__ CUtensorMap tm_pb,
                             const __grid_constant__ CUtensorMap tm_b2, const Params p) {
  static_assert(BN % 16 == 0 && BN >= 64 && BN <= 256, "pair UMMA N for M = 256");
  constexpr int BN_HALF = PairTile<BN>::BN_HALF;
  constexpr int B_BYTES = PairTile<BN>::B_BYTES;
  constexpr int STAGE_BYTES = PairTile<BN>::STAGE_BYTES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * A_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(sB + STAGES * B_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + NUM_ACC;
  uint64_t* done = tempty + NUM_ACC;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int* never = reinterpret_cast<int*>(tmem_slot + 2);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < NUM_ACC; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 8);  // 4 epilogue warps x 2 CTAs (only the leader's is used)
    }
    mbar_init(done, 1);
    *abort_flag = 0;
    *never = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_a);
    tma_prefetch_desc(&tm_b);
    if (p.lora_k) {
      tma_prefetch_desc(&tm_pa);
      tma_prefetch_desc(&tm_pb);
    }
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();  // barrier inits and TMEM allocation visible to the peer
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_launch_dependents();
  pdl_wait();  // the set-up above overlaps the previous kernel; A, B and C are touched after it

  const int num_tiles = p.num_m * p.num_n;
  const int cluster_id = blockIdx.x >> 1;
  const int num_clusters = gridDim.x >> 1;
  const int num_kb = p.k / BK;
  const int total_kb = num_kb + (p.lora_k ? 1 : 0);

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t armed = 0, armed_parity = 0;
      for (int tile = cluster_id; tile < num_tiles; tile += num_clusters) {
        int mb, nb;
        tile_coords(tile, p.num_m, p.num_n, p.group_m, mb, nb);
        const int row_a = mb * 2 * BM + static_cast<int>(rank) * BM;
        // gate/up in one launch: CTA 0 of the pair loads gate rows, CTA 1 up
        // rows, so both CTAs' accumulators hold matching gate | up columns
        const bool two_b = p.epi == GEMM_EPI_SWIGLU;
        const int row_b = two_b ? nb * BN_HALF : nb * BN + static_cast<int>(rank) * BN_HALF;
        const CUtensorMap* tmb = two_b && rank == 1 ? &tm_b2 : &tm_b;
        bool ok = true;
        for (int kb = 0; kb < total_kb; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag, p.status)) { ok = false; break; }
          const uint32_t bar = mapa_shared(smem_u32(&full[stage]), 0);
          if (leader) {
            mbar_arrive_expect_tx(&full[stage], 2 * STAGE_BYTES);
            armed |= 1u << stage;
            armed_parity = (armed_parity & ~(1u << stage)) | (phase << stage);
          }
          if (kb < num_kb) {
            tma_load_2d_pair(sA + stage * A_BYTES, &tm_a, bar, kb * BK, row_a);
            tma_load_2d_pair(sB + stage * B_BYTES, tmb, bar, kb * BK, row_b);
          } else {
            tma_load_2d_pair(sA + stage * A_BYTES, &tm_pa, bar, 0, row_a);
            tma_load_2d_pair(sB + stage * B_BYTES, &tm_pb, bar, 0, row_b);
          }
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
      }
      // The leader's full barriers count both CTAs' bytes: never leave a bulk copy in flight.
      if (leader)
        for (int s = 0; s < STAGES; ++s)
          if (armed & (1u << s)) mbar_wait(&full[s], (armed_parity >> s) & 1u, never, p.status);
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      const uint32_t idesc = umma_idesc_bf16_f32(2 * BM, BN);
      // Shared-memory descriptors of stage 0; a stage is A_BYTES / B_BYTES further
      // (the 14-bit start-address field counts 16-byte units; shared addresses <
      // 256 KB never carry out of it).  Built once: rebuilding two descriptors
      // per MMA made this single issuing thread, not the tensor pipe, the
      // bottleneck (~72% tensor activity per clock).
      const uint64_t a_desc0 = umma_smem_desc_sw128(smem_u32(sA));
      const uint64_t b_desc0 = umma_smem_desc_sw128(smem_u32(sB));
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int tile = cluster_id; tile < num_tiles && ok; tile += num_clusters) {
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1, abort_flag, p.status)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * ACC_STRIDE;
        for (int kb = 0; kb < total_kb; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort_flag, p.status)) { ok = false; break; }
          tc_fence_after();
          const uint64_t ad = a_desc0 + static_cast<uint64_t>(stage * (A_BYTES >> 4));
          const uint64_t bd = b_desc0 + static_cast<uint64_t>(stage * (B_BYTES >> 4));
          const int nk = kb < num_kb ? BK / 16 : p.lora_k / 16;
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk)  // +32 bytes = +2 in the start-address field
            if (kk < nk) umma_bf16_ss_pair(d_tmem, ad + 2 * kk, bd + 2 * kk, idesc, (kb > 0 || kk > 0) ? 1u : 0u);
          umma_commit_pair(&empty[stage]);
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        umma_commit_pair(&tfull[acc]);
        if (++acc == NUM_ACC) { acc = 0; acc_phase ^= 1; }
      }
      umma_commit_pair(done);
    }
  } else {
    const int quarter = warp & 3;
    const uint32_t tempty_leader[NUM_ACC] = {mapa_shared(smem_u32(&tempty[0]), 0),
                                             mapa_shared(smem_u32(&tempty[1]), 0)};
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int tile = cluster_id; tile < num_tiles; tile += num_clusters) {
      int mb, nb;
      tile_coords(tile, p.num_m, p.num_n, p.group_m, mb, nb);
      if (!mbar_wait(&tfull[acc], acc_phase, abort_flag, p.status)) break;
      tc_fence_after();
      const int row = mb * 2 * BM + static_cast<int>(rank) * BM + quarter * 32 + lane;
      const bool row_ok = row < p.m;
      __nv_bfloat16* crow = p.c + (int64_t)row * p.ldc;
      const __nv_bfloat16* arow = p.c_add ? p.c_add + (int64_t)row * p.ldc_add : nullptr;
      const uint32_t tlane = static_cast<uint32_t>(quarter * 32) << 16;
      if (p.epi == GEMM_EPI_SWIGLU) {
        // TMEM columns [0, 128): gate, [128, 256): up, for act columns nb*128 ..
#pragma unroll 1
        for (int chunk = 0; chunk < BN_HALF / 32; ++chunk) {
          const int col0 = nb * BN_HALF + chunk * 32;
          uint32_t rg[32], ru[32];
          tmem_ld_32x32b_x32(tmem_base + tlane + static_cast<uint32_t>(acc * ACC_STRIDE + chunk * 32), rg);
          tmem_ld_32x32b_x32(tmem_base + tlane + static_cast<uint32_t>(acc * ACC_STRIDE + BN_HALF + chunk * 32), ru);
          tmem_ld_wait();
          if (row_ok) {
#pragma unroll
            for (int v = 0; v < 4; ++v) {
              const int col = col0 + v * 8;
              uint32_t gp[4], up[4], ap[4];
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                gp[j] = pack_bf16x2(__uint_as_float(rg[v * 8 + 2 * j]), __uint_as_float(rg[v * 8 + 2 * j + 1]));
                up[j] = pack_bf16x2(__uint_as_float(ru[v * 8 + 2 * j]), __uint_as_float(ru[v * 8 + 2 * j + 1]));
                const float2 g2 = unpack_bf16x2(gp[j]), u2 = unpack_bf16x2(up[j]);
                ap[j] = pack_bf16x2(swiglu_elem(g2.x, u2.x), swiglu_elem(g2.y, u2.y));
              }
              const int64_t o = (int64_t)row * p.ldc + col;
              *reinterpret_cast<uint4*>(p.c + o) = make_uint4(ap[0], ap[1], ap[2], ap[3]);
              if (p.aux0) *reinterpret_cast<uint4*>(p.aux0 + o) = make_uint4(gp[0], gp[1], gp[2], gp[3]);
              if (p.aux1) *reinterpret_cast<uint4*>(p.aux1 + o) = make_uint4(up[0], up[1], up[2], up[3]);
            }
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) remote_arrive(tempty_leader[acc]);
        if (++acc == NUM_ACC) { acc = 0; acc_phase ^= 1; }
        continue;
      }
#pragma unroll 1
      for (int chunk = 0; chunk < (BN + 31) / 32; ++chunk) {
        const int col0 = nb * BN + chunk * 32;
        if (col0 >= p.n) break;  // warp-uniform
        uint32_t r[32];
        // (a last chunk of 16 reads 16 columns past the tile, inside the allocation)
        tmem_ld_32x32b_x32(tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) +
                               static_cast<uint32_t>(acc * ACC_STRIDE + chunk * 32),
                           r);
        tmem_ld_wait();
        if (row_ok) {
#pragma unroll
          for (int v = 0; v < 4; ++v) {
            const int col = col0 + v * 8;
            if (col < p.n && chunk * 32 + v * 8 < BN) {
              float f[8];
#pragma unroll
              for (int j = 0; j < 8; ++j) f[j] = __uint_as_float(r[v * 8 + j]);
              if (p.epi == GEMM_EPI_DSWIGLU) {
                // d = bf16(product); gate / up rows at the same columns
                const int64_t o = (int64_t)row * p.ldc + col;
                const uint4 gq = *reinterpret_cast<const uint4*>(p.src0 + o);
                const uint4 uq = *reinterpret_cast<const uint4*>(p.src1 + o);
                const uint32_t ga[4] = {gq.x, gq.y, gq.z, gq.w}, ua[4] = {uq.x, uq.y, uq.z, uq.w};
                uint32_t dg[4], du[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                  const float2 d2 = unpack_bf16x2(pack_bf16x2(f[2 * j], f[2 * j + 1]));
                  const float2 g2 = unpack_bf16x2(ga[j]), u2 = unpack_bf16x2(ua[j]);
                  float g0, g1, u0, u1;
                  swiglu_grad_elem(d2.x, g2.x, u2.x, g0, u0);
                  swiglu_grad_elem(d2.y, g2.y, u2.y, g1, u1);
                  dg[j] = pack_bf16x2(g0, g1);
                  du[j] = pack_bf16x2(u0, u1);
                }
                *reinterpret_cast<uint4*>(crow + col) = make_uint4(dg[0], dg[1], dg[2], dg[3]);
                *reinterpret_cast<uint4*>(p.aux0 + o) = make_uint4(du[0], du[1], du[2], du[3]);
                continue;
              }
              if (p.bias) add_bf16x8(f, p.bias + col);
              if (arow) add_bf16x8(f, arow + col);
              uint4 o;
              o.x = pack_bf16x2(f[0], f[1]);
              o.y = pack_bf16x2(f[2], f[3]);
              o.z = pack_bf16x2(f[4], f[5]);
              o.w = pack_bf16x2(f[6], f[7]);
              *reinterpret_cast<uint4*>(crow + col) = o;
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) remote_arrive(tempty_leader[acc]);
      if (++acc == NUM_ACC) { acc = 0; acc_phase ^= 1; }
    }
  }

  __syncthreads();
  // Every MMA of the pair reads both CTAs' shared memory: wait for the
  // leader's final commit (multicast to both CTAs) before either CTA leaves.
  if (warp == 1 && lane == 0) mbar_wait(done, 0, never, p.status);
  __syncwarp();
  cluster_sync();  // the peer's shared memory and barriers stay alive until both are done
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, TMEM_COLS);
  }
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (fn == nullptr) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) !=
            cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return nullptr;
    fn = reinterpret_cast<EncodeTiledFn>(ptr);
  }
  return fn;
}

bool make_tmap(CUtensorMap* m, const void* base, int64_t rows, int64_t cols, int64_t ld,
               int box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld * 2)};
  cuuint32_t box[2] = {64u, static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1u, 1u};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box,
                  estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r == CUDA_ERROR_INVALID_CONTEXT && bind_primary_context())
    r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

constexpr int kMaxDev = 64;

}  // namespace

// Pair tile width: 256 unless a narrower one finishes the grid in less tile
// time (waves of num_sms / 2 pairs x width); the SwiGLU epilogues need 256.
// FITQ_GEMM_BN2 forces one of the built widths.
int pick_bn_pair(const GemmArgs& g, int num_sms) {
  static const int widths[] = {256, 192, 160, 144, 128};
  if (g.epi != GEMM_EPI_PLAIN) return 256;
  const char* e = getenv("FITQ_GEMM_BN2");
  if (e != nullptr)
    for (int w : widths)
      if (atoi(e) == w) return w;
  const int64_t mt = (g.m + 2 * BM - 1) / (2 * BM), pairs = num_sms / 2;
  // Only grids of under two waves at 256 columns lose much to the last wave;
  // larger ones keep the wide tile (fewer A re-reads, better MMA efficiency).
  if (mt * ((g.n + 255) / 256) >= 2 * pairs) return 256;
  int best = 256;
  int64_t best_cost = -1;
  for (int w : widths) {
    const int64_t tiles = mt * ((g.n + w - 1) / w);
    const int64_t cost = (tiles + pairs - 1) / pairs * w;
    if (best_cost < 0 || cost < best_cost) {  // ties keep the wider tile
      best = w;
      best_cost = cost;
    }
  }
  return best;
}

template <int BN>
int launch_gemm_bf16_tn_2cta_bn(const GemmArgs& g, cudaStream_t st, int num_sms);

int launch_gemm_bf16_tn_2cta(const GemmArgs& g, cudaStream_t st, int num_sms) {
  switch (pick_bn_pair(g, num_sms)) {
    case 192: return launch_gemm_bf16_tn_2cta_bn<192>(g, st, num_sms);
    case 160: return launch_gemm_bf16_tn_2cta_bn<160>(g, st, num_sms);
    case 144: return launch_gemm_bf16_tn_2cta_bn<144>(g, st, num_sms);
    case 128: return launch_gemm_bf16_tn_2cta_bn<128>(g, st, num_sms);
    default: return launch_gemm_bf16_tn_2cta_bn<256>(g, st, num_sms);
  }
}

template <int BN>
int launch_gemm_bf16_tn_2cta_bn(const GemmArgs& g, cudaStream_t st, int num_sms) {
  constexpr int BN_HALF = PairTile<BN>::BN_HALF;
  constexpr size_t SMEM_BYTES = PairTile<BN>::SMEM_BYTES;
  CUtensorMap ta, tb, tpa, tpb, tb2;
  const bool two_b = g.epi == GEMM_EPI_SWIGLU;
  if (g.epi != GEMM_EPI_PLAIN && BN != 256) return FITQ_ERR_UNSUPPORTED;
  if (two_b && (g.n % BN_HALF != 0 || g.b2 == nullptr || g.lora_k != 0 || g.bias || g.c_add))
    return FITQ_ERR_UNSUPPORTED;
  if (g.epi == GEMM_EPI_DSWIGLU && (!g.src0 || !g.src1 || !g.aux0 || g.bias || g.c_add))
    return FITQ_ERR_UNSUPPORTED;
  if (!make_tmap(&ta, g.a, g.m, g.k, g.lda, BM)) return FITQ_ERR_CUDA;
  if (!make_tmap(&tb, g.b, g.n, g.k, g.ldb, BN_HALF)) return FITQ_ERR_CUDA;
  if (two_b) {
    if (!make_tmap(&tb2, g.b2, g.n, g.k, g.ldb, BN_HALF)) return FITQ_ERR_CUDA;
  } else {
    tb2 = tb;
  }
  if (g.lora_k) {
    if (!make_tmap(&tpa, g.pa, g.m, 64, 64, BM)) return FITQ_ERR_CUDA;
    if (!make_tmap(&tpb, g.pb, g.n, 64, 64, BN_HALF)) return FITQ_ERR_CUDA;
  } else {
    tpa = ta;
    tpb = tb;
  }
  Params p;
  p.c = static_cast<__nv_bfloat16*>(g.c);
  p.c_add = static_cast<const __nv_bfloat16*>(g.c_add);
  p.bias = static_cast<const __nv_bfloat16*>(g.bias);
  p.ldc = g.ldc;
  p.ldc_add = g.ldc_add;
  p.m = static_cast<int>(g.m);
  p.n = static_cast<int>(g.n);
  p.k = static_cast<int>(g.k);
  p.lora_k = g.lora_k;
  p.num_m = static_cast<int>((g.m + 2 * BM - 1) / (2 * BM));
  p.num_n = two_b ? static_cast<int>(g.n / BN_HALF) : static_cast<int>((g.n + BN - 1) / BN);
  p.status = g.status;
  p.epi = g.epi;
  p.src0 = static_cast<const __nv_bfloat16*>(g.src0);
  p.src1 = static_cast<const __nv_bfloat16*>(g.src1);
  p.aux0 = static_cast<__nv_bfloat16*>(g.aux0);
  p.aux1 = static_cast<__nv_bfloat16*>(g.aux1);
  {
    const char* gm = getenv("FITQ_GEMM_GROUP_M");
    // 16 pair tiles (4,096 rows) per group when there are many N tiles: half
    // the DRAM re-reads of B (gate/up forward +5% at M = 32,768); 8 otherwise
    // (k/v: 4 N tiles, 8 measured better).
    p.group_m = gm ? atoi(gm) : (p.num_n >= 16 ? 2 * GROUP_M : GROUP_M);
    if (p.group_m < 1) p.group_m = GROUP_M;
  }
  static bool attr_set[kMaxDev] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= kMaxDev) return FITQ_ERR_NO_DEVICE;
  if (!attr_set[dev]) {
    if (cudaFuncSetAttribute(gemm_bf16_tn_2cta_kernel<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(SMEM_BYTES)) != cudaSuccess)
      return FITQ_ERR_CUDA;
    attr_set[dev] = true;
  }
  const int tiles = p.num_m * p.num_n;
  const int clusters = tiles < num_sms / 2 ? tiles : num_sms / 2;
  const double flops = 2.0 * static_cast<double>(g.m) * static_cast<double>(g.n) *
                       static_cast<double>(g.k + g.lora_k) * (two_b ? 2.0 : 1.0);
  const int slot = timing_begin(st, flops);
  launch_pdl(gemm_bf16_tn_2cta_kernel<BN>, dim3(2 * clusters), dim3(NUM_THREADS), SMEM_BYTES, st, ta, tb, tpa, tpb,
             tb2, p);
  note_launch();
  timing_end(slot, st);
  return launch_result();
}

}  // namespace fitq
