// NF4 dequant fused into the tcgen05 GEMM on CTA pairs (cta_group::2):
// 256 x 256 output tile per pair, each CTA decoding its own half of the
// weight operand from the packed codes straight into its shared memory.
//
//   forward (trans = 0):  C[M, N] = X[M, K] . W_deq[N, K]^T   (+ LoRA K-block)
//   dX      (trans = 1):  C[M, K] = dY[M, N] . W_deq[N, K]     (+ LoRA K-block)
//
// W_deq is bitsandbytes' dequant of the NF4 weight, bit for bit:
//   absmax_b = fl(fl(nested_quant_map[code_b] * nested_absmax[b / 256]) + offset)
//   w        = bf16_rn(fl(quant_map[nibble] * absmax_b))
// (two rounded fp32 operations, no FMA), the values FitLLM's Linear4bit
// forward (fitllm/forward.py:680-686) and MatMul4Bit.backward
// (fitllm/backward.py:234) obtain before their cuBLAS call.
//
// A cluster of two CTAs on neighbouring SMs shares one MMA (M = 256, N = 256):
// CTA r holds rows [128r, 128r+128) of the A tile and columns [128r, 128r+128)
// of the weight operand in its own shared memory.  Per CTA (480 threads):
//   warp 0       TMA of the CTA's A half (128 x 64 bf16, 128-byte swizzle),
//                completing on the leader's "full" barrier (no multicast).
//   warp 1       TMEM (512 columns: two 128 x 256 fp32 accumulators); in the
//                leader, one lane issues tcgen05.mma.cta_group::2 and commits
//                to both CTAs' barriers.
//   warps 2-5    epilogue of the CTA's 128 rows (double-buffered TMEM).
//   warp 6       TMA of the packed bytes of the CTA's weight half (4 KB per
//                K step) into an 8-stage ring of its own.
//   warps 7-14   decoders, two groups of four warps taking alternate K steps:
//                a thread decodes one 64-weight NF4 block of one W row once
//                the slot's previous MMAs retired (absmax inputs fetched two
//                of its steps ahead): the block's 16-entry table
//                bf16(fl(qm[i] * absmax)) as two byte planes of four
//                registers, four weights per pair of prmt lookups, one
//                128-byte operand row in the 128-byte-swizzled layout (K-major
//                rows of W for the forward, MN-major for dX), then
//                fence.proxy.async and one arrive per warp on the LEADER's
//                "decoded" barrier (release at cluster scope).
// The LoRA term s.(P.Q^T) is one extra K-block whose operands come by TMA.
// Every mbarrier wait is bounded (common.cuh).
#include <cstdlib>

#include "common.cuh"
#include "kernels.cuh"
#include "nf4_decode.cuh"
#include "pair.cuh"

namespace fitq {
namespace {

constexpr int BM = 128;       // A rows per CTA (pair tile: 256)
constexpr int BN_HALF = 128;  // weight-operand columns per CTA
constexpr int BN = 256;       // output columns per pair tile
constexpr int BK = 64;
constexpr int PSTAGES = 8;    // packed-byte ring
constexpr int A_BYTES = BM * BK * 2;       // 16 KB per 256-row pair sub-tile
constexpr int B_BYTES = BN_HALF * BK * 2;  // 16 KB decoded (or the LoRA Q half)
constexpr int P_BYTES = BN_HALF * BK / 2;  // 4 KB packed NF4
#ifndef FITQ_NF4_DEC_GROUPS
#define FITQ_NF4_DEC_GROUPS 4
#endif
constexpr int DEC_GROUPS = FITQ_NF4_DEC_GROUPS;  // groups of four decoder warps, taking K steps in turn
constexpr int NUM_DEC_WARPS = 4 * DEC_GROUPS;
constexpr int DEC_WARP0 = 7;
constexpr int NUM_THREADS = (DEC_WARP0 + NUM_DEC_WARPS) * 32;
constexpr int TMEM_COLS = 512;
constexpr int GROUP_M = 8;  // pair tiles (256 rows) per raster group
constexpr uint32_t MN_LBO = 1024;  // MN-major operand: bytes between 64-column atoms
constexpr uint32_t MN_SBO = 2048;  // ... and between 8-row K groups
// MSUB 256-row pair sub-tiles share each decoded weight tile: MSUB = 1 keeps
// two TMEM accumulators (epilogue overlaps the next tile), MSUB = 2 halves the
// decode work per FLOP with one 512-column accumulator set.
template <int MSUB>
struct Cfg {
  static constexpr int STAGES = MSUB == 1 ? 5 : 4;  // A + decoded-B ring
  static constexpr int NUM_ACC = MSUB == 1 ? 2 : 1;
  static constexpr int ACC_COLS = MSUB * BN;
  static constexpr int A_STAGE = MSUB * A_BYTES;
  static constexpr size_t SMEM =
      1024 + STAGES * (A_STAGE + B_BYTES) + PSTAGES * P_BYTES + 256 * 4 + 512;
  static_assert(SMEM <= 232448, "shared memory budget");
  static_assert(NUM_ACC * ACC_COLS <= TMEM_COLS, "tensor memory budget");
};

struct Params {
  __nv_bfloat16* c;
  const __nv_bfloat16* c_add;
  const __nv_bfloat16* bias;
  int64_t ldc, ldc_add;
  int m, n, k;  // GEMM: C[m, n] = A[m, k] . B[n, k]^T
  int lora_k;
  int num_m, num_n, group_m;  // in pair tiles
  int trans;
  int w_kb;  // NF4 blocks per W row
  const uint8_t* codes;
  const float* nabs;
  const float* absmax_f32;
  const float* qm;
  const float* nqm;
  float offset;
  int* status;
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

// One decoder group's K steps (tile, kb) in order -- the steps whose running
// index has the group's parity, LoRA steps excluded -- for the two-ahead
// prefetch of the absmax inputs.
struct DecCursor {
  int tile, kb, it, nb;
};

__device__ __forceinline__ bool dec_next(DecCursor& c, int group, int num_tiles, int stride,
                                         int total_kb, int num_kb, const Params& p) {
  while (true) {
    if (++c.kb == total_kb) {
      c.kb = 0;
      c.tile += stride;
      if (c.tile >= num_tiles) return false;
      int mb;
      tile_coords(c.tile, p.num_m, p.num_n, p.group_m, mb, c.nb);
    }
    ++c.it;
    if (c.it % DEC_GROUPS == group && c.kb < num_kb) return true;
  }
}

template <int MSUB>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(NUM_THREADS, 1)
    gemm_nf4_2cta_kernel(const __grid_constant__ CUtensorMap tm_a,
                         const __grid_constant__ CUtensorMap tm_p,
                         const __grid_constant__ CUtensorMap tm_pa,
                         const __grid_constant__ CUtensorMap tm_pb, const Params p) {
  constexpr int STAGES = Cfg<MSUB>::STAGES;
  constexpr int NUM_ACC = Cfg<MSUB>::NUM_ACC;
  constexpr int ACC_COLS = Cfg<MSUB>::ACC_COLS;
  constexpr int A_STAGE = Cfg<MSUB>::A_STAGE;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* sA = smem;
  uint8_t* sB = sA + STAGES * A_STAGE;
  uint8_t* sP = sB + STAGES * B_BYTES;
  float* s_nqm = reinterpret_cast<float*>(sP + PSTAGES * P_BYTES);
  uint64_t* full = reinterpret_cast<uint64_t*>(s_nqm + 256);  // both A halves landed (leader)
  uint64_t* bfull = full + STAGES;                             // both B halves decoded (leader)
  uint64_t* empty = bfull + STAGES;                            // the slot's MMAs retired (both)
  uint64_t* pfull = empty + STAGES;                            // packed bytes landed (own)
  uint64_t* pempty = pfull + PSTAGES;                          // packed bytes consumed (own)
  uint64_t* tfull = pempty + PSTAGES;
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
      mbar_init(&bfull[s], 2 * 4);  // the four warps of the step's group x 2 CTAs
      mbar_init(&empty[s], 1);
    }
    for (int s = 0; s < PSTAGES; ++s) {
      mbar_init(&pfull[s], 1);
      mbar_init(&pempty[s], 4);
    }
    for (int a = 0; a < NUM_ACC; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 8);  // 4 epilogue warps x 2 CTAs (the leader's is used)
    }
    mbar_init(done, 1);
    *abort_flag = 0;
    *never = 0;
    fence_mbar_init();
  }
  if (p.nqm != nullptr && threadIdx.x < 256) s_nqm[threadIdx.x] = p.nqm[threadIdx.x];
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_a);
    tma_prefetch_desc(&tm_p);
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
  cluster_sync();  // barrier inits, the nested map and TMEM allocation visible to the pair
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
    // ------------------------------------------------ A (and LoRA) producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t armed = 0, armed_parity = 0;
      for (int tile = cluster_id; tile < num_tiles; tile += num_clusters) {
        int mb, nb;
        tile_coords(tile, p.num_m, p.num_n, p.group_m, mb, nb);
        const int row_a = mb * MSUB * 2 * BM + static_cast<int>(rank) * BM;
        const int row_b = nb * BN + static_cast<int>(rank) * BN_HALF;
        bool ok = true;
        for (int kb = 0; kb < total_kb; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag, p.status)) { ok = false; break; }
          const uint32_t bar = mapa_shared(smem_u32(&full[stage]), 0);
          const bool lora = kb >= num_kb;
          if (leader) {
            mbar_arrive_expect_tx(&full[stage], lora ? 2 * (A_STAGE + B_BYTES) : 2 * A_STAGE);
            armed |= 1u << stage;
            armed_parity = (armed_parity & ~(1u << stage)) | (phase << stage);
          }
#pragma unroll
          for (int h = 0; h < MSUB; ++h)  // sub-tile h: rows + 256 h
            tma_load_2d_pair(sA + stage * A_STAGE + h * A_BYTES, lora ? &tm_pa : &tm_a, bar,
                             lora ? 0 : kb * BK, row_a + h * 2 * BM);
          if (lora) tma_load_2d_pair(sB + stage * B_BYTES, &tm_pb, bar, 0, row_b);
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
      }
      // the leader's full barriers count both CTAs' bytes: no bulk copy left in flight
      if (leader)
        for (int s = 0; s < STAGES; ++s)
          if (armed & (1u << s)) mbar_wait(&full[s], (armed_parity >> s) & 1u, never, p.status);
    }
  } else if (warp == 6) {
    // ------------------------------------------------ packed-byte producer (own half)
    if (lane == 0) {
      int ps = 0;
      uint32_t pph = 0;
      uint32_t armed = 0, armed_parity = 0;
      for (int tile = cluster_id; tile < num_tiles; tile += num_clusters) {
        int mb, nb;
        tile_coords(tile, p.num_m, p.num_n, p.group_m, mb, nb);
        const int col0 = nb * BN + static_cast<int>(rank) * BN_HALF;  // first operand column
        bool ok = true;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&pempty[ps], pph ^ 1, abort_flag, p.status)) { ok = false; break; }
          armed |= 1u << ps;
          armed_parity = (armed_parity & ~(1u << ps)) | (pph << ps);
          mbar_arrive_expect_tx(&pfull[ps], P_BYTES);
          if (p.trans)  // W rows kb*64.., bytes of W columns col0..col0+127
            tma_load_2d(sP + ps * P_BYTES, &tm_p, &pfull[ps], col0 / 2, kb * BK);
          else  // W rows col0.., bytes of W columns kb*64..
            tma_load_2d(sP + ps * P_BYTES, &tm_p, &pfull[ps], kb * (BK / 2), col0);
          if (++ps == PSTAGES) { ps = 0; pph ^= 1; }
        }
        if (!ok) break;
      }
      for (int s = 0; s < PSTAGES; ++s)
        if (armed & (1u << s)) mbar_wait(&pfull[s], (armed_parity >> s) & 1u, never, p.status);
    }
  } else if (warp == 1) {
    // ------------------------------------------------ MMA issuer (leader)
    if (lane == 0 && leader) {
      const uint32_t idesc_w = umma_idesc_bf16_f32(2 * BM, BN) | (p.trans ? (1u << 16) : 0u);
      const uint32_t idesc_k = umma_idesc_bf16_f32(2 * BM, BN);
      const uint64_t a_desc0 = umma_smem_desc_sw128(smem_u32(sA));
      const uint64_t b_desc0 = umma_smem_desc_sw128(smem_u32(sB));
      const uint64_t b_desc0_mn = umma_smem_desc_sw128_mn(smem_u32(sB), MN_LBO, MN_SBO);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int tile = cluster_id; tile < num_tiles && ok; tile += num_clusters) {
        if (!mbar_wait_cluster(&tempty[acc], acc_phase ^ 1, abort_flag, p.status)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * ACC_COLS;
        for (int kb = 0; kb < total_kb; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort_flag, p.status) ||
              !mbar_wait_cluster(&bfull[stage], phase, abort_flag, p.status)) { ok = false; break; }
          tc_fence_after();
          const bool lora = kb >= num_kb;
          const int nk = lora ? p.lora_k / 16 : BK / 16;
          const bool mn = p.trans && !lora;
          const uint64_t ad = a_desc0 + static_cast<uint64_t>(stage * (A_STAGE >> 4));
          const uint64_t bd = (mn ? b_desc0_mn : b_desc0) + static_cast<uint64_t>(stage * (B_BYTES >> 4));
          const uint32_t idesc = lora ? idesc_k : idesc_w;
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            if (kk < nk) {
              // K step of 16: +32 bytes inside the swizzle row (K-major), or two
              // 8-row K groups further (MN-major)
              const uint64_t b = bd + (mn ? static_cast<uint64_t>(kk * (2 * MN_SBO >> 4)) : 2ull * kk);
#pragma unroll
              for (int h = 0; h < MSUB; ++h)
                umma_bf16_ss_pair(d_tmem + h * BN, ad + h * (A_BYTES >> 4) + 2 * kk, b, idesc,
                                  (kb > 0 || kk > 0) ? 1u : 0u);
            }
          }
          umma_commit_pair(&empty[stage]);
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        umma_commit_pair(&tfull[acc]);
        if (++acc == NUM_ACC) { acc = 0; acc_phase ^= 1; }
      }
      umma_commit_pair(done);
    }
  } else if (warp < 6) {
    // ------------------------------------------------ epilogue (this CTA's 128 rows)
    const int quarter = warp & 3;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int tile = cluster_id; tile < num_tiles; tile += num_clusters) {
      int mb, nb;
      tile_coords(tile, p.num_m, p.num_n, p.group_m, mb, nb);
      if (!mbar_wait(&tfull[acc], acc_phase, abort_flag, p.status)) break;
      tc_fence_after();
#pragma unroll 1
      for (int h = 0; h < MSUB; ++h) {
        const int row = (mb * MSUB + h) * 2 * BM + static_cast<int>(rank) * BM + quarter * 32 + lane;
        const bool row_ok = row < p.m;
        __nv_bfloat16* crow = p.c + (int64_t)row * p.ldc;
        const __nv_bfloat16* arow = p.c_add ? p.c_add + (int64_t)row * p.ldc_add : nullptr;
#pragma unroll 1
        for (int chunk = 0; chunk < BN / 32; ++chunk) {
          const int col0 = nb * BN + chunk * 32;
          uint32_t r[32];
          tmem_ld_32x32b_x32(tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) +
                                 static_cast<uint32_t>(acc * ACC_COLS + h * BN + chunk * 32),
                             r);
          tmem_ld_wait();
          if (row_ok) {
#pragma unroll
            for (int v = 0; v < 4; ++v) {
              const int col = col0 + v * 8;
              float f[8];
#pragma unroll
              for (int j = 0; j < 8; ++j) f[j] = __uint_as_float(r[v * 8 + j]);
#pragma unroll
              for (int src = 0; src < 2; ++src) {
                const __nv_bfloat16* add = src == 0 ? (p.bias ? p.bias + col : nullptr)
                                                    : (arow ? arow + col : nullptr);
                if (add) {
                  const uint4 q = *reinterpret_cast<const uint4*>(add);
                  const uint32_t qa[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
                  for (int j = 0; j < 4; ++j) {
                    const float2 t = unpack_bf16x2(qa[j]);
                    f[2 * j] += t.x;
                    f[2 * j + 1] += t.y;
                  }
                }
              }
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
      if (lane == 0) remote_arrive(mapa_shared(smem_u32(&tempty[acc]), 0));
      if (++acc == NUM_ACC) { acc = 0; acc_phase ^= 1; }
    }
  } else {
    // ------------------------------------------------ decoders (own weight half)
    const int dw = warp - DEC_WARP0;
    const int group = dw >> 2;
    const int u = (dw & 3) * 32 + lane;  // unit: one 64-weight NF4 block of one W row
    uint64_t qm[8];
    nf4_load_qm_pairs(p.qm, qm);
    // forward: W row col0 + u, block kb -> operand row u (K-major);
    // dX: W row kb*64 + u/2, block col0/64 + (u & 1) -> K-row u/2, MN atom u & 1.
    const int r_local = p.trans ? (u >> 1) : u;
    const int jb = p.trans ? (u & 1) : 0;
    const uint32_t src_off = p.trans ? static_cast<uint32_t>(r_local * 64 + jb * 32)
                                     : static_cast<uint32_t>(u * 32);
    const uint32_t dst_off = p.trans ? static_cast<uint32_t>((r_local >> 3) * MN_SBO + jb * MN_LBO +
                                                             (r_local & 7) * 128)
                                     : static_cast<uint32_t>(u * 128);
    const uint32_t swz = static_cast<uint32_t>(r_local & 7);
    const bool plain = p.absmax_f32 != nullptr;
    auto fetch = [&](const DecCursor& c, uint32_t& code, float& scale) {
      const int col0 = c.nb * BN + static_cast<int>(rank) * BN_HALF;
      const int64_t wrow = p.trans ? (int64_t)c.kb * BK + r_local : (int64_t)col0 + u;
      const int64_t b = wrow * p.w_kb + (p.trans ? col0 / 64 + jb : c.kb);
      if (plain) {
        code = 0;
        scale = __ldg(p.absmax_f32 + b);
      } else {
        code = __ldg(p.codes + b);
        scale = __ldg(p.nabs + (b >> 8));
      }
    };
    DecCursor la{cluster_id, -1, -1, 0};
    {
      int mb;
      tile_coords(la.tile, p.num_m, p.num_n, p.group_m, mb, la.nb);
    }
    uint32_t code0 = 0, code1 = 0;
    float sc0 = 0.f, sc1 = 0.f;
    const bool have0 = dec_next(la, group, num_tiles, num_clusters, total_kb, num_kb, p);
    if (have0) fetch(la, code0, sc0);
    bool have1 = have0 && dec_next(la, group, num_tiles, num_clusters, total_kb, num_kb, p);
    if (have1) fetch(la, code1, sc1);

    int it = 0, pit = 0;  // K steps, packed stages
    bool ok = true;
    for (int tile = cluster_id; tile < num_tiles && ok; tile += num_clusters) {
      for (int kb = 0; kb < total_kb; ++kb, ++it) {
        const bool lora = kb >= num_kb;
        const int my_pit = pit;
        if (!lora) ++pit;
        if (it % DEC_GROUPS != group) continue;
        const int stage = it % STAGES;
        const uint32_t phase = static_cast<uint32_t>(it / STAGES) & 1u;
        // the B slot is free once the MMAs that read it last have retired
        if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag, p.status)) { ok = false; break; }
        if (!lora) {
          const float am = plain ? sc0 : __fadd_rn(__fmul_rn(s_nqm[code0], sc0), p.offset);
          code0 = code1;
          sc0 = sc1;
          if (have1) {
            have1 = dec_next(la, group, num_tiles, num_clusters, total_kb, num_kb, p);
            if (have1) fetch(la, code1, sc1);
          }
          const int ps = my_pit % PSTAGES;
          const uint32_t pph = static_cast<uint32_t>(my_pit / PSTAGES) & 1u;
          if (!mbar_wait(&pfull[ps], pph, abort_flag, p.status)) { ok = false; break; }
          nf4_decode_row(sP + ps * P_BYTES + src_off, sB + stage * B_BYTES + dst_off, swz, qm, am);
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) mbar_arrive(&pempty[ps]);  // bytes consumed
        }
        __syncwarp();
        if (lane == 0) remote_arrive(mapa_shared(smem_u32(&bfull[stage]), 0));
      }
    }
  }

  __syncthreads();
  // every MMA of the pair reads both CTAs' shared memory: wait for the leader's
  // final commit (multicast to both CTAs) before either CTA leaves
  if (warp == 1 && lane == 0) mbar_wait(done, 0, never, p.status);
  __syncwarp();
  cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, TMEM_COLS);
  }
}

bool make_tmap_bf16(CUtensorMap* m, const void* base, int64_t rows, int64_t cols, int64_t ld,
                    int box_rows) {
  return encode_tmap_2d(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, base, static_cast<uint64_t>(cols),
                        static_cast<uint64_t>(rows), static_cast<uint64_t>(ld) * 2, 64u,
                        static_cast<uint32_t>(box_rows), CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B);
}


// 512-row tiles when there are enough of them to occupy the pairs (half the
// decode work per FLOP, epilogue not overlapped); FITQ_NF4_MSUB=1|2 forces one.
bool use_msub2(int64_t m, int64_t n, int num_sms) {
  const char* e = getenv("FITQ_NF4_MSUB");
  if (e != nullptr && (e[0] == '1' || e[0] == '2')) return e[0] == '2';
  const int64_t tiles2 = ((m + 511) / 512) * (n / BN);
  return tiles2 >= num_sms;  // at least two 512-row tiles per pair
}

}  // namespace

bool gemm_nf4_2cta_supported(const Nf4Args& w, int trans) {
  const int64_t n = trans ? w.k_in : w.n_out;
  const int64_t k = trans ? w.n_out : w.k_in;
  return n % BN == 0 && k % BK == 0 && w.k_in % 64 == 0 && n < (1ll << 31) && k < (1ll << 31) &&
         (reinterpret_cast<uintptr_t>(w.packed) & 15u) == 0;
}

int launch_gemm_nf4_2cta(const Nf4GemmArgs& g, cudaStream_t st, int num_sms) {
  const Nf4Args& w = g.w;
  if (!gemm_nf4_2cta_supported(w, g.trans)) return FITQ_ERR_UNSUPPORTED;
  const int64_t n = g.trans ? w.k_in : w.n_out;
  const int64_t k = g.trans ? w.n_out : w.k_in;
  CUtensorMap ta, tp, tpa, tpb;
  if (!make_tmap_bf16(&ta, g.a, g.m, k, g.lda, BM)) return FITQ_ERR_CUDA;
  // packed bytes as a [N_w rows, K_w / 2 bytes] uint8 matrix
  if (!encode_tmap_2d(&tp, CU_TENSOR_MAP_DATA_TYPE_UINT8, w.packed, static_cast<uint64_t>(w.k_in / 2),
                      static_cast<uint64_t>(w.n_out), static_cast<uint64_t>(w.k_in / 2),
                      g.trans ? BN_HALF / 2 : BK / 2, g.trans ? BK : BN_HALF,
                      CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B))
    return FITQ_ERR_CUDA;
  if (g.lora_k) {
    if (!make_tmap_bf16(&tpa, g.pa, g.m, 64, 64, BM)) return FITQ_ERR_CUDA;
    if (!make_tmap_bf16(&tpb, g.pb, n, 64, 64, BN_HALF)) return FITQ_ERR_CUDA;
  } else {
    tpa = ta;
    tpb = ta;
  }
  Params p;
  p.c = static_cast<__nv_bfloat16*>(g.c);
  p.c_add = static_cast<const __nv_bfloat16*>(g.c_add);
  p.bias = static_cast<const __nv_bfloat16*>(g.bias);
  p.ldc = g.ldc;
  p.ldc_add = g.ldc_add;
  p.m = static_cast<int>(g.m);
  p.n = static_cast<int>(n);
  p.k = static_cast<int>(k);
  p.lora_k = g.lora_k;
  const int msub = use_msub2(g.m, n, num_sms) ? 2 : 1;
  p.num_m = static_cast<int>((g.m + 2 * BM * msub - 1) / (2 * BM * msub));
  p.num_n = static_cast<int>(n / BN);
  p.trans = g.trans;
  p.w_kb = static_cast<int>(w.k_in / 64);
  p.codes = w.absmax_code;
  p.nabs = w.nested_absmax;
  p.absmax_f32 = w.absmax_f32;
  p.qm = w.quant_map;
  p.nqm = w.absmax_f32 ? nullptr : w.nested_quant_map;
  p.offset = w.offset;
  p.status = g.status;
  {
    const char* gm = getenv("FITQ_GEMM_GROUP_M");
    p.group_m = gm ? atoi(gm) : (p.num_n >= 16 ? 2 * GROUP_M : GROUP_M);
    if (p.group_m < 1) p.group_m = GROUP_M;
  }
  // once per (device, kernel), under the helper's lock
  if (!(msub == 1 ? set_smem_limit(gemm_nf4_2cta_kernel<1>, static_cast<int>(Cfg<1>::SMEM))
                  : set_smem_limit(gemm_nf4_2cta_kernel<2>, static_cast<int>(Cfg<2>::SMEM))))
    return FITQ_ERR_CUDA;
  const int tiles = p.num_m * p.num_n;
  const int clusters = tiles < num_sms / 2 ? tiles : num_sms / 2;
  const double flops = 2.0 * static_cast<double>(g.m) * static_cast<double>(n) *
                       static_cast<double>(k + g.lora_k);
  const int slot = timing_begin(st, flops);
  if (msub == 1)
    launch_pdl(gemm_nf4_2cta_kernel<1>, dim3(2 * clusters), dim3(NUM_THREADS), Cfg<1>::SMEM, st, ta, tp, tpa,
               tpb, p);
  else
    launch_pdl(gemm_nf4_2cta_kernel<2>, dim3(2 * clusters), dim3(NUM_THREADS), Cfg<2>::SMEM, st, ta, tp, tpa,
               tpb, p);
  note_launch();
  timing_end(slot, st);
  return launch_result();
}

}  // namespace fitq
