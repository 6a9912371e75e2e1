// tcgen05 / TMEM / TMA GEMM for sm_100a:  C = A.B^T (+ LoRA block) (+ C_add).
//
// Persistent, warp-specialised CTA (192 threads, one CTA per SM):
//   warp 0     TMA producer: A[128x64] and B[256x64] bf16 tiles, 128-byte
//              swizzle, into a 4-stage shared-memory ring (48 KB per stage).
//   warp 1     owns the TMEM allocation (512 columns = two 128x256 fp32
//              accumulators) and issues tcgen05.mma kind::f16 from one lane.
//   warps 2-5  epilogue: tcgen05.ld 32 lanes x 32 columns, bf16 convert,
//              optional residual add, global store.  Double-buffered TMEM lets
//              the epilogue of tile i overlap the main loop of tile i+1.
// The LoRA term P.Q^T (P[M,r], Q[N,r], r <= 64) is one extra k-block fed from
// two more tensor maps and accumulated into the same TMEM accumulator, so the
// adapter costs r/16 extra MMA instructions per tile and no extra pass.
// Every mbarrier wait is bounded (common.cuh); no TMA multicast is used.
#include <cstdlib>

#include <cstdio>

#include "common.cuh"
#include "kernels.cuh"

namespace fitq {
namespace {

// Tile width BN is a template parameter: 256 by default; narrower tiles
// (a multiple of 16) when the tile count of the 256-wide grid would leave
// most of a wave idle (few rows: 512 x 5120 has 80 tiles of 128 x 256 on 148
// SMs, but 144 tiles of 128 x 144).  The two accumulators sit 256 TMEM
// columns apart whatever BN is.
constexpr int BM = 128, BK = 64;
constexpr int STAGES = 4;
constexpr int A_BYTES = BM * BK * 2;
constexpr int NUM_THREADS = 192;
constexpr int NUM_ACC = 2;
constexpr int ACC_STRIDE = 256;
constexpr int TMEM_COLS = 512;
constexpr int GROUP_M = 16;  // M-tiles (128 rows) per raster group
template <int BN>
constexpr int b_bytes() { return BN * BK * 2; }
template <int BN>
constexpr size_t smem_bytes() { return 1024 /*align slack*/ + STAGES * (A_BYTES + b_bytes<BN>()) + 256; }

struct Params {
  __nv_bfloat16* c;
  const __nv_bfloat16* c_add;
  const __nv_bfloat16* bias;  // [N], broadcast over rows (may be null)
  int64_t ldc, ldc_add;
  int m, n, k;
  int lora_k;
  int num_m, num_n;
  int group_m;  // M-tiles per raster group (L2 reuse of the B tiles)
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

template <int BN>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    gemm_bf16_tn_kernel(const __grid_constant__ CUtensorMap tm_a,
                        const __grid_constant__ CUtensorMap tm_b,
                        const __grid_constant__ CUtensorMap tm_pa,
                        const __grid_constant__ CUtensorMap tm_pb, const Params p) {
  static_assert(BN % 16 == 0 && BN >= 64 && BN <= 256, "UMMA N for M = 128");
  pdl_launch_dependents();
  constexpr int B_BYTES = b_bytes<BN>();
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
  int* never = reinterpret_cast<int*>(tmem_slot + 2);  // stays 0: teardown waits run to the limit

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < NUM_ACC; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 4);
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
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_wait();  // the set-up above overlaps the previous kernel; A, B and C are touched after it

  const int num_tiles = p.num_m * p.num_n;
  const int num_kb = p.k / BK;
  const int total_kb = num_kb + (p.lora_k ? 1 : 0);

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t armed = 0, armed_parity = 0;  // per-stage bit: armed / parity of last arm
      for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
        int mb, nb;
        tile_coords(tile, p.num_m, p.num_n, p.group_m, mb, nb);
        bool ok = true;
        for (int kb = 0; kb < total_kb; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag, p.status)) { ok = false; break; }
          mbar_arrive_expect_tx(&full[stage], A_BYTES + B_BYTES);
          armed |= 1u << stage;
          armed_parity = (armed_parity & ~(1u << stage)) | (phase << stage);
          if (kb < num_kb) {
            tma_load_2d(sA + stage * A_BYTES, &tm_a, &full[stage], kb * BK, mb * BM);
            tma_load_2d(sB + stage * B_BYTES, &tm_b, &full[stage], kb * BK, nb * BN);
          } else {
            tma_load_2d(sA + stage * A_BYTES, &tm_pa, &full[stage], 0, mb * BM);
            tma_load_2d(sB + stage * B_BYTES, &tm_pb, &full[stage], 0, nb * BN);
          }
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
      }
      // Never leave a bulk copy in flight: wait for the last arm of each stage.
      for (int s = 0; s < STAGES; ++s)
        if (armed & (1u << s)) mbar_wait(&full[s], (armed_parity >> s) & 1u, never, p.status);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = umma_idesc_bf16_f32(BM, BN);
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
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
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
            if (kk < nk) umma_bf16_ss(d_tmem, ad + 2 * kk, bd + 2 * kk, idesc, (kb > 0 || kk > 0) ? 1u : 0u);
          umma_commit(&empty[stage]);
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        umma_commit(&tfull[acc]);
        if (++acc == NUM_ACC) { acc = 0; acc_phase ^= 1; }
      }
      // All issued MMAs must retire before TMEM is released.
      umma_commit(done);
      mbar_wait(done, 0, never, p.status);
    }
  } else {
    const int quarter = warp & 3;  // TMEM lanes 32*quarter .. +31
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
      int mb, nb;
      tile_coords(tile, p.num_m, p.num_n, p.group_m, mb, nb);
      if (!mbar_wait(&tfull[acc], acc_phase, abort_flag, p.status)) break;
      tc_fence_after();
      const int row = mb * BM + quarter * 32 + lane;
      const bool row_ok = row < p.m;
      __nv_bfloat16* crow = p.c + (int64_t)row * p.ldc;
      const __nv_bfloat16* arow = p.c_add ? p.c_add + (int64_t)row * p.ldc_add : nullptr;
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
      if (++acc == NUM_ACC) { acc = 0; acc_phase ^= 1; }
    }
  }

  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

// ---------------------------------------------------------------- host side
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

// 2-D bf16 row-major [rows, cols] with row pitch ld (elements); box = 64 cols x box_rows.
bool make_tmap(CUtensorMap* m, const void* base, int64_t rows, int64_t cols, int64_t ld,
               int box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld * 2)};
  cuuint32_t box[2] = {64u, static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1u, 1u};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides,
                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r == CUDA_ERROR_INVALID_CONTEXT && bind_primary_context())
    r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

}  // namespace

bool encode_tmap_2d(CUtensorMap* m, CUtensorMapDataType dtype, const void* base, uint64_t inner,
                    uint64_t outer, uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer,
                    CUtensorMapSwizzle swizzle, CUtensorMapL2promotion l2) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(inner), static_cast<cuuint64_t>(outer)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(row_bytes)};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1u, 1u};
  CUresult r = fn(m, dtype, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, l2, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r == CUDA_ERROR_INVALID_CONTEXT && bind_primary_context())
    r = fn(m, dtype, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
           swizzle, l2, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    char msg[256];
    snprintf(msg, sizeof(msg),
             "cuTensorMapEncodeTiled = %d (dtype %d, base %p, dims %llu x %llu, row %llu B, box %u x %u, "
             "swizzle %d, l2 %d)",
             static_cast<int>(r), static_cast<int>(dtype), base, static_cast<unsigned long long>(inner),
             static_cast<unsigned long long>(outer), static_cast<unsigned long long>(row_bytes), box_inner,
             box_outer, static_cast<int>(swizzle), static_cast<int>(l2));
    note_launch_detail(msg);
  }
  return r == CUDA_SUCCESS;
}

// Tile width: 256 unless a narrower one finishes the grid in less tile time
// (waves x width, one CTA per SM); FITQ_GEMM_BN forces one of the built widths.
int pick_bn(int64_t m, int64_t n, int num_sms) {
  static const int widths[] = {256, 192, 160, 144, 128};
  const char* e = getenv("FITQ_GEMM_BN");
  if (e != nullptr)
    for (int w : widths)
      if (atoi(e) == w) return w;
  const int64_t mt = (m + BM - 1) / BM;
  // Only grids of under two waves at 256 columns lose much to the last wave;
  // larger ones keep the wide tile (fewer A re-reads, better MMA efficiency).
  if (mt * ((n + 255) / 256) >= 2 * num_sms) return 256;
  int best = 256;
  int64_t best_cost = -1;
  for (int w : widths) {
    const int64_t tiles = mt * ((n + w - 1) / w);
    const int64_t cost = (tiles + num_sms - 1) / num_sms * w;
    if (best_cost < 0 || cost < best_cost) {  // ties keep the wider tile
      best = w;
      best_cost = cost;
    }
  }
  return best;
}

template <int BN>
int launch_gemm_bf16_tn_bn(const GemmArgs& g, cudaStream_t st, int num_sms);

int launch_gemm_bf16_tn(const GemmArgs& g, cudaStream_t st, int num_sms) {
  switch (pick_bn(g.m, g.n, num_sms)) {
    case 192: return launch_gemm_bf16_tn_bn<192>(g, st, num_sms);
    case 160: return launch_gemm_bf16_tn_bn<160>(g, st, num_sms);
    case 144: return launch_gemm_bf16_tn_bn<144>(g, st, num_sms);
    case 128: return launch_gemm_bf16_tn_bn<128>(g, st, num_sms);
    default: return launch_gemm_bf16_tn_bn<256>(g, st, num_sms);
  }
}

template <int BN>
int launch_gemm_bf16_tn_bn(const GemmArgs& g, cudaStream_t st, int num_sms) {
  constexpr size_t SMEM_BYTES = smem_bytes<BN>();
  CUtensorMap ta, tb, tpa, tpb;
  if (!make_tmap(&ta, g.a, g.m, g.k, g.lda, BM)) return FITQ_ERR_CUDA;
  if (!make_tmap(&tb, g.b, g.n, g.k, g.ldb, BN)) return FITQ_ERR_CUDA;
  if (g.lora_k) {
    if (!make_tmap(&tpa, g.pa, g.m, 64, 64, BM)) return FITQ_ERR_CUDA;
    if (!make_tmap(&tpb, g.pb, g.n, 64, 64, BN)) return FITQ_ERR_CUDA;
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
  p.num_m = static_cast<int>((g.m + BM - 1) / BM);
  p.num_n = static_cast<int>((g.n + BN - 1) / BN);
  p.status = g.status;
  {
    const char* gm = getenv("FITQ_GEMM_GROUP_M");
    p.group_m = gm ? atoi(gm) : GROUP_M;
    if (p.group_m < 1) p.group_m = GROUP_M;
  }
  if (!set_smem_limit(gemm_bf16_tn_kernel<BN>, static_cast<int>(SMEM_BYTES))) return FITQ_ERR_CUDA;
  const int tiles = p.num_m * p.num_n;
  const int grid = tiles < num_sms ? tiles : num_sms;
  const double flops = 2.0 * static_cast<double>(g.m) * static_cast<double>(g.n) *
                       static_cast<double>(g.k + g.lora_k);
  const int slot = timing_begin(st, flops);
  launch_pdl(gemm_bf16_tn_kernel<BN>, dim3(grid), dim3(NUM_THREADS), SMEM_BYTES, st, ta, tb, tpa, tpb, p);
  note_launch();
  timing_end(slot, st);
  return launch_result();
}

int launch_gemm(const GemmArgs& g, cudaStream_t st, int num_sms) {
  if (g.epi != GEMM_EPI_PLAIN) return launch_gemm_bf16_tn_2cta(g, st, num_sms);  // pair-only epilogues
  const char* v = getenv("FITQ_GEMM_VARIANT");
  bool pair;
  if (v && v[0] == '1') {
    pair = false;
  } else if (v && v[0] == '2') {
    pair = true;
  } else {
    // Pair tiles need enough of them for ~4 waves of 74 clusters.  Shapes with
    // K >= 4N (down_proj forward, gate/up dX: N = 5120, K = 27648) run faster
    // on the one-CTA kernel under the 1 kW power cap (measured at M = 32,768:
    // 1.23 vs 1.13 PFLOP/s), the others on the pair kernel (gate/up forward
    // 1.25 vs 1.24, q 1.23 vs 1.19, k/v 1.21 vs 1.16).
    const int64_t tiles2 = ((g.m + 255) / 256) * ((g.n + 255) / 256);
    pair = tiles2 >= 4 * static_cast<int64_t>(num_sms / 2) && g.k < 4 * g.n;
  }
  return pair ? launch_gemm_bf16_tn_2cta(g, st, num_sms) : launch_gemm_bf16_tn(g, st, num_sms);
}

}  // namespace fitq
