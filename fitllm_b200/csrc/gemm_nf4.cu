// NF4 dequant fused into the tcgen05 GEMM: the weight operand is decoded from
// the packed 4-bit codes straight into shared memory, never written to HBM.
//
//   forward (trans = 0):  C[M, N] = X[M, K] . W_deq[N, K]^T   (+ LoRA K-block)
//   dX      (trans = 1):  C[M, K] = dY[M, N] . W_deq[N, K]     (+ LoRA K-block)
//
// W_deq is bitsandbytes' dequant of the NF4 weight, bit for bit:
//   absmax_b = fl(fl(nested_quant_map[code_b] * nested_absmax[b / 256]) + offset)
//   w        = bf16_rn(fl(quant_map[nibble] * absmax_b))
// (two rounded fp32 operations, no FMA), as FitLLM's Linear4bit forward
// (fitllm/forward.py:680-686) and MatMul4Bit.backward (fitllm/backward.py:234)
// obtain it before their cuBLAS call.
//
// Persistent, warp-specialised CTA (480 threads, one per SM), tile 256 x 128:
//   warp 0       TMA of the A tile (256 x 64 bf16, 128-byte swizzle) into a
//                4-stage ring that also holds the decoded B tiles.
//   warp 6       TMA of the packed weight bytes (4 KB per stage, unswizzled)
//                into their own 8-stage ring, so the codes are in shared
//                memory long before their B slot frees up.
//   warp 1       owns TMEM (512 columns: two buffers x two 128 x 128 fp32
//                accumulators) and issues tcgen05.mma kind::f16 from one lane:
//                two M = 128, N = 128 MMAs per K step share the decoded B tile,
//                so every weight is decoded once per 256 rows of A.
//   warps 2-5    epilogue (tcgen05.ld, bias / residual add, bf16 stores),
//                overlapping the next tile's main loop (double-buffered TMEM).
//   warps 7-14   decoders, two groups of four warps taking alternate K
//                steps; a thread decodes one 64-weight NF4 block of one W row
//                once the slot's previous MMAs retired (its absmax inputs
//                fetched two of its steps earlier): it builds the block's
//                16-entry table of bf16 values
//                bf16(fl(qm[i] * absmax)) as two byte planes of four registers,
//                then looks up four weights per pair of prmt instructions and
//                writes the 128-byte operand row in the 128-byte-swizzled
//                layout the MMA reads: K-major rows of W for the forward,
//                MN-major (W's K contiguous) for dX.  fence.proxy.async, then
//                one arrive per warp on the stage's "decoded" barrier.
// The LoRA term s.(P.Q^T) is one extra K-block whose both operands come by TMA
// (bf16, pitch 64) into the same accumulators.  Every mbarrier wait is bounded
// (common.cuh); no TMA multicast is used.
#include <cstdlib>

#include "common.cuh"
#include "kernels.cuh"
#include "nf4_decode.cuh"

namespace fitq {
namespace {

constexpr int BM = 256;  // A rows per tile: two 128-row UMMA sub-tiles
constexpr int BN = 128;
constexpr int BK = 64;
constexpr int STAGES = 4;   // A + decoded-B ring
constexpr int PSTAGES = 8;  // packed-byte ring (runs ahead of the decoders)
constexpr int A_BYTES = BM * BK * 2;  // 32 KB
constexpr int B_BYTES = BN * BK * 2;  // 16 KB decoded (or the LoRA Q tile)
constexpr int P_BYTES = BN * BK / 2;  // 4 KB packed NF4
constexpr int NUM_DEC_WARPS = 8;      // 256 threads: half an NF4 block each per stage
constexpr int DEC_WARP0 = 7;
constexpr int NUM_THREADS = (DEC_WARP0 + NUM_DEC_WARPS) * 32;
constexpr int TMEM_COLS = 512;
constexpr int GROUP_M = 8;  // M-tiles (256 rows) per raster group
// MN-major operand (dX): 8 K-rows x 64 MN elements = one 1 KB swizzle atom;
// the two MN atoms of a K group are adjacent, K groups follow each other.
constexpr uint32_t MN_LBO = 1024;  // bytes between MN atoms
constexpr uint32_t MN_SBO = 2048;  // bytes between 8-row K groups
constexpr size_t SMEM_BYTES = 1024 /*align*/ + STAGES * (A_BYTES + B_BYTES) + PSTAGES * P_BYTES +
                               256 * 4 /*nested map*/ + 512 /*barriers*/;
static_assert(SMEM_BYTES <= 232448, "shared memory budget");

struct Params {
  __nv_bfloat16* c;
  const __nv_bfloat16* c_add;
  const __nv_bfloat16* bias;
  int64_t ldc, ldc_add;
  int m, n, k;  // GEMM: C[m, n] = A[m, k] . B[n, k]^T
  int lora_k;
  int num_m, num_n, group_m;
  int trans;
  int w_kb;  // NF4 blocks per W row (W's K / 64)
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

// Walks one decoder group's iterations (tile, kb) in order: the K steps of
// the CTA's tiles whose running index has the group's parity, LoRA steps
// excluded.  Used to fetch each block's absmax inputs two iterations early.
struct DecCursor {
  int tile, kb, it, nb;
};

__device__ __forceinline__ bool dec_next(DecCursor& c, int group, int num_tiles, int total_kb,
                                         int num_kb, const Params& p) {
  while (true) {
    if (++c.kb == total_kb) {
      c.kb = 0;
      c.tile += gridDim.x;
      if (c.tile >= num_tiles) return false;
      int mb;
      tile_coords(c.tile, p.num_m, p.num_n, p.group_m, mb, c.nb);
    }
    ++c.it;
    if ((c.it & 1) == group && c.kb < num_kb) return true;
  }
}

__global__ void __launch_bounds__(NUM_THREADS, 1)
    gemm_nf4_kernel(const __grid_constant__ CUtensorMap tm_a,
                    const __grid_constant__ CUtensorMap tm_p,
                    const __grid_constant__ CUtensorMap tm_pa,
                    const __grid_constant__ CUtensorMap tm_pb, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* sA = smem;
  uint8_t* sB = sA + STAGES * A_BYTES;
  uint8_t* sP = sB + STAGES * B_BYTES;
  float* s_nqm = reinterpret_cast<float*>(sP + PSTAGES * P_BYTES);
  uint64_t* full = reinterpret_cast<uint64_t*>(s_nqm + 256);  // A (or LoRA P+Q) landed
  uint64_t* bfull = full + STAGES;                             // B decoded
  uint64_t* empty = bfull + STAGES;                            // MMAs of the slot retired
  uint64_t* pfull = empty + STAGES;                            // packed bytes landed
  uint64_t* pempty = pfull + PSTAGES;                          // packed bytes read
  uint64_t* tfull = pempty + PSTAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* done = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int* never = reinterpret_cast<int*>(tmem_slot + 2);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&bfull[s], NUM_DEC_WARPS / 2);  // one arrive per warp of the stage's group
      mbar_init(&empty[s], 1);
    }
    for (int s = 0; s < PSTAGES; ++s) {
      mbar_init(&pfull[s], 1);
      mbar_init(&pempty[s], NUM_DEC_WARPS / 2);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 4);
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
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_launch_dependents();
  pdl_wait();  // the set-up above overlaps the previous kernel; A, B and C are touched after it

  const int num_tiles = p.num_m * p.num_n;
  const int num_kb = p.k / BK;
  const int total_kb = num_kb + (p.lora_k ? 1 : 0);

  if (warp == 0) {
    // ------------------------------------------------ A (and LoRA) producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t armed = 0, armed_parity = 0;
      for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
        int mb, nb;
        tile_coords(tile, p.num_m, p.num_n, p.group_m, mb, nb);
        bool ok = true;
        for (int kb = 0; kb < total_kb; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag, p.status)) { ok = false; break; }
          armed |= 1u << stage;
          armed_parity = (armed_parity & ~(1u << stage)) | (phase << stage);
          if (kb < num_kb) {
            mbar_arrive_expect_tx(&full[stage], A_BYTES);
            tma_load_2d(sA + stage * A_BYTES, &tm_a, &full[stage], kb * BK, mb * BM);
          } else {
            mbar_arrive_expect_tx(&full[stage], A_BYTES + B_BYTES);
            tma_load_2d(sA + stage * A_BYTES, &tm_pa, &full[stage], 0, mb * BM);
            tma_load_2d(sB + stage * B_BYTES, &tm_pb, &full[stage], 0, nb * BN);
          }
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
      }
      for (int s = 0; s < STAGES; ++s)
        if (armed & (1u << s)) mbar_wait(&full[s], (armed_parity >> s) & 1u, never, p.status);
    }
  } else if (warp == 6) {
    // ------------------------------------------------ packed-byte producer
    if (lane == 0) {
      int ps = 0;
      uint32_t pph = 0;
      uint32_t armed = 0, armed_parity = 0;
      for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
        int mb, nb;
        tile_coords(tile, p.num_m, p.num_n, p.group_m, mb, nb);
        bool ok = true;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&pempty[ps], pph ^ 1, abort_flag, p.status)) { ok = false; break; }
          armed |= 1u << ps;
          armed_parity = (armed_parity & ~(1u << ps)) | (pph << ps);
          mbar_arrive_expect_tx(&pfull[ps], P_BYTES);
          if (p.trans)  // W rows kb*64.., bytes of W columns nb*128..
            tma_load_2d(sP + ps * P_BYTES, &tm_p, &pfull[ps], nb * (BN / 2), kb * BK);
          else  // W rows nb*128.., bytes of W columns kb*64..
            tma_load_2d(sP + ps * P_BYTES, &tm_p, &pfull[ps], kb * (BK / 2), nb * BN);
          if (++ps == PSTAGES) { ps = 0; pph ^= 1; }
        }
        if (!ok) break;
      }
      for (int s = 0; s < PSTAGES; ++s)
        if (armed & (1u << s)) mbar_wait(&pfull[s], (armed_parity >> s) & 1u, never, p.status);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc_w = umma_idesc_bf16_f32(128, BN) | (p.trans ? (1u << 16) : 0u);
      const uint32_t idesc_k = umma_idesc_bf16_f32(128, BN);
      const uint64_t a_desc0 = umma_smem_desc_sw128(smem_u32(sA));
      const uint64_t b_desc0 = umma_smem_desc_sw128(smem_u32(sB));
      const uint64_t b_desc0_mn = umma_smem_desc_sw128_mn(smem_u32(sB), MN_LBO, MN_SBO);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1, abort_flag, p.status)) break;
        tc_fence_after();
        const uint32_t d0 = tmem_base + acc * 2 * BN;
        for (int kb = 0; kb < total_kb; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort_flag, p.status) ||
              !mbar_wait(&bfull[stage], phase, abort_flag, p.status)) { ok = false; break; }
          tc_fence_after();
          const uint64_t ad = a_desc0 + static_cast<uint64_t>(stage * (A_BYTES >> 4));
          const bool lora = kb >= num_kb;
          const int nk = lora ? p.lora_k / 16 : BK / 16;
          const bool mn = p.trans && !lora;
          const uint64_t bd = (mn ? b_desc0_mn : b_desc0) + static_cast<uint64_t>(stage * (B_BYTES >> 4));
          const uint32_t idesc = lora ? idesc_k : idesc_w;
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            if (kk < nk) {
              // K step of 16: +32 bytes inside the swizzle row (K-major), or
              // two 8-row K groups further (MN-major)
              const uint64_t b = bd + (mn ? static_cast<uint64_t>(kk * (2 * MN_SBO >> 4)) : 2ull * kk);
              const uint32_t accum = (kb > 0 || kk > 0) ? 1u : 0u;
              umma_bf16_ss(d0, ad + 2 * kk, b, idesc, accum);
              umma_bf16_ss(d0 + BN, ad + (A_BYTES / 2 >> 4) + 2 * kk, b, idesc, accum);
            }
          }
          umma_commit(&empty[stage]);
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        umma_commit(&tfull[acc]);
        if (++acc == 2) { acc = 0; acc_phase ^= 1; }
      }
      umma_commit(done);
      mbar_wait(done, 0, never, p.status);
    }
  } else if (warp < 6) {
    const int quarter = warp & 3;  // TMEM lanes 32*quarter .. +31
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
      int mb, nb;
      tile_coords(tile, p.num_m, p.num_n, p.group_m, mb, nb);
      if (!mbar_wait(&tfull[acc], acc_phase, abort_flag, p.status)) break;
      tc_fence_after();
#pragma unroll 1
      for (int h = 0; h < 2; ++h) {
        const int row = mb * BM + h * 128 + quarter * 32 + lane;
        const bool row_ok = row < p.m;
        __nv_bfloat16* crow = p.c + (int64_t)row * p.ldc;
        const __nv_bfloat16* arow = p.c_add ? p.c_add + (int64_t)row * p.ldc_add : nullptr;
#pragma unroll 1
        for (int chunk = 0; chunk < BN / 32; ++chunk) {
          const int col0 = nb * BN + chunk * 32;
          uint32_t r[32];
          tmem_ld_32x32b_x32(tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) +
                                 static_cast<uint32_t>((acc * 2 + h) * BN + chunk * 32),
                             r);
          tmem_ld_wait();
          if (row_ok) {
#pragma unroll
            for (int v = 0; v < 4; ++v) {
              const int col = col0 + v * 8;
              float f[8];
#pragma unroll
              for (int j = 0; j < 8; ++j) f[j] = __uint_as_float(r[v * 8 + j]);
              if (p.bias) {
                const uint4 q = *reinterpret_cast<const uint4*>(p.bias + col);
                const uint32_t qa[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                  const float2 t = unpack_bf16x2(qa[j]);
                  f[2 * j] += t.x;
                  f[2 * j + 1] += t.y;
                }
              }
              if (arow) {
                const uint4 q = *reinterpret_cast<const uint4*>(arow + col);
                const uint32_t qa[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                  const float2 t = unpack_bf16x2(qa[j]);
                  f[2 * j] += t.x;
                  f[2 * j + 1] += t.y;
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
      if (lane == 0) mbar_arrive(&tempty[acc]);
      if (++acc == 2) { acc = 0; acc_phase ^= 1; }
    }
  } else {
    // ------------------------------------------------------------ decoders
    const int dw = warp - DEC_WARP0;
    const int group = dw >> 2;           // takes the K steps of this parity
    const int u = (dw & 3) * 32 + lane;  // unit: one 64-weight NF4 block of one W row
    uint64_t qm[8];
    nf4_load_qm_pairs(p.qm, qm);
    // Unit geometry within the stage.
    //   forward: W row nb*128 + u, block kb; operand row u (K-major).
    //   dX:      W row kb*64 + u/2, block nb*2 + (u & 1); K-row u/2 of the
    //            MN-major operand, MN atom (u & 1).
    const int r_local = p.trans ? (u >> 1) : u;
    const int jb = p.trans ? (u & 1) : 0;
    const uint32_t src_off = p.trans ? static_cast<uint32_t>(r_local * 64 + jb * 32)
                                     : static_cast<uint32_t>(u * 32);
    const uint32_t dst_off = p.trans ? static_cast<uint32_t>((r_local >> 3) * MN_SBO + jb * MN_LBO +
                                                             (r_local & 7) * 128)
                                     : static_cast<uint32_t>(u * 128);
    const uint32_t swz = static_cast<uint32_t>(r_local & 7);
    const bool plain = p.absmax_f32 != nullptr;
    // absmax inputs of this thread's block in K step (nb, kb)
    auto block_of = [&](int nb, int kb) -> int64_t {
      const int64_t wrow = p.trans ? (int64_t)kb * BK + r_local : (int64_t)nb * BN + u;
      return wrow * p.w_kb + (p.trans ? nb * 2 + jb : kb);
    };
    auto fetch = [&](const DecCursor& c, uint32_t& code, float& scale) {
      const int64_t b = block_of(c.nb, c.kb);
      if (plain) {
        code = 0;
        scale = __ldg(p.absmax_f32 + b);
      } else {
        code = __ldg(p.codes + b);
        scale = __ldg(p.nabs + (b >> 8));
      }
    };
    // two-deep prefetch of the absmax inputs over this group's K steps
    DecCursor la{static_cast<int>(blockIdx.x), -1, -1, 0};
    {
      int mb;
      tile_coords(la.tile, p.num_m, p.num_n, p.group_m, mb, la.nb);
    }
    uint32_t code0 = 0, code1 = 0;
    float sc0 = 0.f, sc1 = 0.f;
    bool have0 = dec_next(la, group, num_tiles, total_kb, num_kb, p);
    if (have0) fetch(la, code0, sc0);
    bool have1 = have0 && dec_next(la, group, num_tiles, total_kb, num_kb, p);
    if (have1) fetch(la, code1, sc1);

    int it = 0, pit = 0;  // K steps (all), packed stages (LoRA steps excluded)
    bool ok = true;
    for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
      for (int kb = 0; kb < total_kb; ++kb, ++it) {
        const bool lora = kb >= num_kb;
        const int my_pit = pit;
        if (!lora) ++pit;
        if ((it & 1) != group) continue;
        const int stage = it % STAGES;
        const uint32_t phase = static_cast<uint32_t>(it / STAGES) & 1u;
        // the B slot is free once the MMAs that read it last have retired
        if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag, p.status)) { ok = false; break; }
        if (!lora) {
          const float am = plain ? sc0 : __fadd_rn(__fmul_rn(s_nqm[code0], sc0), p.offset);
          code0 = code1;
          sc0 = sc1;
          if (have1) {
            have1 = dec_next(la, group, num_tiles, total_kb, num_kb, p);
            if (have1) fetch(la, code1, sc1);
          }
          const int ps = my_pit % PSTAGES;
          const uint32_t pph = static_cast<uint32_t>(my_pit / PSTAGES) & 1u;
          if (!mbar_wait(&pfull[ps], pph, abort_flag, p.status)) { ok = false; break; }
          nf4_decode_row(sP + ps * P_BYTES + src_off, sB + stage * B_BYTES + dst_off, swz, qm, am);
          fence_proxy_async_smem();
          // the packed slot is released only after its bytes were consumed
          __syncwarp();
          if (lane == 0) mbar_arrive(&pempty[ps]);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&bfull[stage]);
      }
    }
  }

  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

bool make_tmap_bf16(CUtensorMap* m, const void* base, int64_t rows, int64_t cols, int64_t ld,
                    int box_rows) {
  return encode_tmap_2d(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, base, static_cast<uint64_t>(cols),
                        static_cast<uint64_t>(rows), static_cast<uint64_t>(ld) * 2, 64u,
                        static_cast<uint32_t>(box_rows), CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B);
}


}  // namespace

bool gemm_nf4_supported(const Nf4Args& w, int trans) {
  const int64_t n = trans ? w.k_in : w.n_out;  // GEMM output columns
  const int64_t k = trans ? w.n_out : w.k_in;  // GEMM reduction
  return n % BN == 0 && k % BK == 0 && w.k_in % 64 == 0 && n < (1ll << 31) && k < (1ll << 31) &&
         (reinterpret_cast<uintptr_t>(w.packed) & 15u) == 0;
}

int launch_gemm_nf4(const Nf4GemmArgs& g, cudaStream_t st, int num_sms) {
  const Nf4Args& w = g.w;
  const char* v = getenv("FITQ_NF4_GEMM");
  const bool one_cta = v != nullptr && v[0] == '1';
  if (!one_cta && gemm_nf4_2cta_supported(w, g.trans)) return launch_gemm_nf4_2cta(g, st, num_sms);
  if (!gemm_nf4_supported(w, g.trans)) return FITQ_ERR_UNSUPPORTED;
  const int64_t n = g.trans ? w.k_in : w.n_out;
  const int64_t k = g.trans ? w.n_out : w.k_in;
  CUtensorMap ta, tp, tpa, tpb;
  if (!make_tmap_bf16(&ta, g.a, g.m, k, g.lda, BM)) return FITQ_ERR_CUDA;
  // packed bytes as a [N_w rows, K_w / 2 bytes] uint8 matrix
  if (!encode_tmap_2d(&tp, CU_TENSOR_MAP_DATA_TYPE_UINT8, w.packed, static_cast<uint64_t>(w.k_in / 2),
                      static_cast<uint64_t>(w.n_out), static_cast<uint64_t>(w.k_in / 2),
                      g.trans ? BN / 2 : BK / 2, g.trans ? BK : BN, CU_TENSOR_MAP_SWIZZLE_NONE,
                      CU_TENSOR_MAP_L2_PROMOTION_L2_256B))
    return FITQ_ERR_CUDA;
  if (g.lora_k) {
    if (!make_tmap_bf16(&tpa, g.pa, g.m, 64, 64, BM)) return FITQ_ERR_CUDA;
    if (!make_tmap_bf16(&tpb, g.pb, n, 64, 64, BN)) return FITQ_ERR_CUDA;
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
  p.num_m = static_cast<int>((g.m + BM - 1) / BM);
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
    p.group_m = gm ? atoi(gm) : GROUP_M;
    if (p.group_m < 1) p.group_m = GROUP_M;
  }
  if (!set_smem_limit(gemm_nf4_kernel, static_cast<int>(SMEM_BYTES))) return FITQ_ERR_CUDA;
  const int tiles = p.num_m * p.num_n;
  const int grid = tiles < num_sms ? tiles : num_sms;
  const double flops = 2.0 * static_cast<double>(g.m) * static_cast<double>(n) *
                       static_cast<double>(k + g.lora_k);
  const int slot = timing_begin(st, flops);
  launch_pdl(gemm_nf4_kernel, dim3(grid), dim3(NUM_THREADS), SMEM_BYTES, st, ta, tp, tpa, tpb, p);
  note_launch();
  timing_end(slot, st);
  return launch_result();
}

}  // namespace fitq
