// Speculative-verify attention over a key/value cache (split-KV flash decoding).
//
// FitLLM verifies draft tokens by re-running the whole prefix through the
// model (fitllm/inference.py:380-397, attention inside fitllm/forward.py's
// layer forward).  With a KV cache the verify step attends T new tokens of
// each sequence to prefix + T cached positions: new token i sees positions
// <= prefix + i (causal among the new tokens, full over the prefix).  That is
// a few query rows against a long cache -- a read of the cache, bounded by
// HBM -- which the general attention kernels tile poorly.
//
// Layouts: q [B, T, H, D] and out [B, T, H, D] bf16 (the q_proj output and
// the o_proj input, no transposes); k_cache, v_cache [B, KVH, cap, D] bf16.
// D = 128.  The G = H / KVH query heads of a KV head and the T new tokens are
// folded into G * T <= 32 query rows (row = head_in_group * T + token), so a
// KV tile is read once for all of them.
//
// verify_attn_kernel: grid (splits, KVH, B), 4 warps.  A CTA walks its range
// of 64-position tiles (cp.async double buffer, XOR-swizzled 16-byte chunks:
// conflict-free ldmatrix).  Per tile, warp w computes S = Q.K^T for positions
// 16w..16w+15 and all 32 rows (mma.sync m16n8k16 bf16, fp32 accumulate), the
// CTA reduces the row maxima through shared memory (online softmax in base 2,
// masked positions get probability exactly 0), writes P (bf16) to shared
// memory, and warp w accumulates O[:, 32w..32w+31] += P.V.  The CTA's
// (O, m, l) go to a workspace; verify_attn_combine_kernel merges the splits
// in split order (deterministic) and writes bf16 out.
#include "common.cuh"
#include "kernels.cuh"

namespace fitq {
namespace {

constexpr int kAttD = 128;
constexpr int kAttRows = 32;    // folded query rows (G * T <= 32)
constexpr int kAttTile = 64;    // KV positions per tile
constexpr int kAttThreads = 128;
constexpr int kAttRowBytes = kAttD * 2;                 // 256 B per Q / K / V row
constexpr int kAttKV = kAttTile * kAttRowBytes;         // 16 KB per K or V tile
constexpr int kAttQ = kAttRows * kAttRowBytes;          // 8 KB
constexpr int kAttP = kAttRows * kAttTile * 2;          // 4 KB
// P lives in the K tile it was computed from (every warp is past S = Q.K^T
// when P is written, and the tile is reloaded only after P.V): 73 KB, so
// three CTAs fit per SM.
constexpr int kAttSmem = kAttQ + 4 * kAttKV + 2 * 4 * kAttRows * 4;  // 73 KB
static_assert(kAttP <= kAttKV, "P must fit in a K tile");
constexpr float kMaskedMax = -1.0e30f;

extern __shared__ __align__(128) uint8_t g_att_smem[];

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                        uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                          uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void mma_bf16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
      "{%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Byte offset of 16-byte chunk c of row r in a [rows][256 B] array: chunk
// index XOR (r & 7) within the row, so the 8 rows of an ldmatrix hit 8 banks.
__device__ __forceinline__ uint32_t swz256(int r, int c) {
  return static_cast<uint32_t>(r * 256 + ((c ^ (r & 7)) << 4));
}
// Same for the [32][128 B] P array.
__device__ __forceinline__ uint32_t swz128(int r, int c) {
  return static_cast<uint32_t>(r * 128 + ((c ^ (r & 7)) << 4));
}

struct AttParams {
  const __nv_bfloat16* q;
  const __nv_bfloat16* k;
  const __nv_bfloat16* v;
  float* o_part;   // [B, KVH, splits, 32, 128]
  float* ml_part;  // [B, KVH, splits, 32, 2]: row max (base-2 scaled) and row sum
  int H, KVH, T, G, rows;  // rows = G * T
  int prefix, len, cap;    // len = prefix + T valid positions
  int splits, tiles_per_split;
  float scale_log2;        // log2(e) / sqrt(D)
};

__global__ void __launch_bounds__(kAttThreads, 3)
    verify_attn_kernel(const AttParams p) {
  const int split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, qd = lane & 3;
  pdl_launch_dependents();
  pdl_wait();  // q and the cache append come from the previous kernel
  const uint32_t s_q = smem_u32(g_att_smem);
  const uint32_t s_k = s_q + kAttQ;              // two K tiles, then two V tiles
  const uint32_t s_v = s_k + 2 * kAttKV;
  float* red_max = reinterpret_cast<float*>(g_att_smem + kAttQ + 4 * kAttKV);
  float* red_sum = red_max + 4 * kAttRows;

  const int tile0 = split * p.tiles_per_split;
  const int ntiles_all = (p.len + kAttTile - 1) / kAttTile;
  int tile1 = tile0 + p.tiles_per_split;
  if (tile1 > ntiles_all) tile1 = ntiles_all;

  // Q rows: row r = head_in_group * T + token -> q[b, token, kvh * G + head_in_group, :];
  // rows >= G * T are zeros.  32 rows x 16 chunks, 4 chunks per thread.
  for (int i = tid; i < kAttRows * 16; i += kAttThreads) {
    const int r = i >> 4, c = i & 15;
    const bool ok = r < p.rows;
    const int hg = ok ? r / p.T : 0, tk = ok ? r % p.T : 0;
    const __nv_bfloat16* src =
        p.q + ((static_cast<int64_t>(b) * p.T + tk) * p.H + kvh * p.G + hg) * kAttD + c * 8;
    cp_async16(s_q + swz256(r, c), src, ok ? 16u : 0u);
  }
  const int64_t kv_base = (static_cast<int64_t>(b) * p.KVH + kvh) * p.cap;
  auto load_tile = [&](int t, int buf) {
    const int pos0 = t * kAttTile;
    for (int i = tid; i < kAttTile * 16; i += kAttThreads) {
      const int r = i >> 4, c = i & 15;
      const bool ok = pos0 + r < p.len;
      const int64_t off = (kv_base + (ok ? pos0 + r : 0)) * kAttD + c * 8;
      cp_async16(s_k + buf * kAttKV + swz256(r, c), p.k + off, ok ? 16u : 0u);
      cp_async16(s_v + buf * kAttKV + swz256(r, c), p.v + off, ok ? 16u : 0u);
    }
  };
  if (tile0 < tile1) load_tile(tile0, 0);
  cp_commit();

  // this thread's rows: 16 mt + g + 8 h, h = 0/1 (fragment rows of both m16 tiles)
  float m_run[2][2], l_run[2][2];
  float o[2][4][4];
#pragma unroll
  for (int mt = 0; mt < 2; ++mt)
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      m_run[mt][h] = kMaskedMax;
      l_run[mt][h] = 0.f;
    }
#pragma unroll
  for (int mt = 0; mt < 2; ++mt)
#pragma unroll
    for (int nt = 0; nt < 4; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) o[mt][nt][e] = 0.f;

  for (int t = tile0; t < tile1; ++t) {
    const int buf = (t - tile0) & 1;
    cp_wait_all();
    __syncthreads();  // tile t (and Q) visible; every warp is done with tile t - 1
    if (t + 1 < tile1) load_tile(t + 1, buf ^ 1);
    cp_commit();
    const uint32_t kb = s_k + buf * kAttKV, vb = s_v + buf * kAttKV;
    const uint32_t s_p = kb;  // P of this tile overwrites its K once S is done
    const int pos0 = t * kAttTile;

    // ---- S = Q.K^T for positions 16 warp .. + 15 (two n8 tiles), all rows
    float s[2][2][4];
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) s[mt][nt][e] = 0.f;
    const int mat = lane >> 3, rr = lane & 7;
#pragma unroll
    for (int ks = 0; ks < kAttD / 16; ++ks) {
      uint32_t k0, k1, k2, k3;  // n8 tile 0: {k0, k1}, n8 tile 1: {k2, k3}
      {
        const int pr = 16 * warp + 8 * (mat >> 1) + rr;
        ldsm_x4(kb + swz256(pr, 2 * ks + (mat & 1)), k0, k1, k2, k3);
      }
#pragma unroll
      for (int mt = 0; mt < 2; ++mt) {
        uint32_t a0, a1, a2, a3;
        const int qr = 16 * mt + 8 * (mat & 1) + rr;
        ldsm_x4(s_q + swz256(qr, 2 * ks + (mat >> 1)), a0, a1, a2, a3);
        mma_bf16(s[mt][0], a0, a1, a2, a3, k0, k1);
        mma_bf16(s[mt][1], a0, a1, a2, a3, k2, k3);
      }
    }

    // ---- mask, scale, row maxima
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int row = 16 * mt + g + 8 * h;
        const int lim = row < p.rows ? p.prefix + row % p.T : -1;  // last visible position
        float mx = kMaskedMax;
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int pos = pos0 + 16 * warp + 8 * nt + 2 * qd + e;
            float& v = s[mt][nt][2 * h + e];
            v = (pos <= lim) ? v * p.scale_log2 : kMaskedMax;
            mx = fmaxf(mx, v);
          }
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
        if (qd == 0) red_max[warp * kAttRows + row] = mx;
      }
    __syncthreads();
    float alpha[2][2];
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int row = 16 * mt + g + 8 * h;
        float mx = fmaxf(fmaxf(red_max[row], red_max[kAttRows + row]),
                         fmaxf(red_max[2 * kAttRows + row], red_max[3 * kAttRows + row]));
        const float m_new = fmaxf(m_run[mt][h], mx);
        alpha[mt][h] = exp2f(m_run[mt][h] - m_new);
        m_run[mt][h] = m_new;
        // probabilities of this warp's positions; masked ones are exactly 0
        float sum = 0.f;
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) {
          float pv[2];
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const float v = s[mt][nt][2 * h + e];
            pv[e] = v > 0.5f * kMaskedMax ? exp2f(v - m_new) : 0.f;
            sum += pv[e];
          }
          const uint32_t pk = pack_bf16x2(pv[0], pv[1]);
          const int col = 16 * warp + 8 * nt + 2 * qd;  // position within the tile
          asm volatile("st.shared.u32 [%0], %1;" ::"r"(s_p + swz128(row, col >> 3) + (col & 7) * 2),
                       "r"(pk)
                       : "memory");
        }
        sum += __shfl_xor_sync(0xffffffffu, sum, 1);
        sum += __shfl_xor_sync(0xffffffffu, sum, 2);
        if (qd == 0) red_sum[warp * kAttRows + row] = sum;
      }
    __syncthreads();
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int row = 16 * mt + g + 8 * h;
        l_run[mt][h] = alpha[mt][h] * l_run[mt][h] + ((red_sum[row] + red_sum[kAttRows + row]) +
                                                      (red_sum[2 * kAttRows + row] +
                                                       red_sum[3 * kAttRows + row]));
#pragma unroll
        for (int nt = 0; nt < 4; ++nt) {
          o[mt][nt][2 * h] *= alpha[mt][h];
          o[mt][nt][2 * h + 1] *= alpha[mt][h];
        }
      }

    // ---- O[:, 32 warp .. + 31] += P.V
#pragma unroll
    for (int ks = 0; ks < kAttTile / 16; ++ks) {
      uint32_t v[4][2];
#pragma unroll
      for (int np = 0; np < 2; ++np) {
        // matrices: (pos 16ks + 8 (mat & 1) .., d chunk 4 warp + 2 np + (mat >> 1))
        const int pr = 16 * ks + 8 * (mat & 1) + rr;
        ldsm_x4_t(vb + swz256(pr, 4 * warp + 2 * np + (mat >> 1)), v[2 * np][0], v[2 * np][1],
                  v[2 * np + 1][0], v[2 * np + 1][1]);
      }
#pragma unroll
      for (int mt = 0; mt < 2; ++mt) {
        uint32_t a0, a1, a2, a3;
        const int pr = 16 * mt + 8 * (mat & 1) + rr;
        ldsm_x4(s_p + swz128(pr, 2 * ks + (mat >> 1)), a0, a1, a2, a3);
#pragma unroll
        for (int nt = 0; nt < 4; ++nt) mma_bf16(o[mt][nt], a0, a1, a2, a3, v[nt][0], v[nt][1]);
      }
    }
  }
  cp_wait_all();

  // ---- partial results of this split
  const int64_t part = (static_cast<int64_t>(b) * p.KVH + kvh) * p.splits + split;
#pragma unroll
  for (int mt = 0; mt < 2; ++mt)
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int row = 16 * mt + g + 8 * h;
      if (row >= p.rows) continue;
      float* orow = p.o_part + (part * kAttRows + row) * kAttD + 32 * warp + 2 * qd;
#pragma unroll
      for (int nt = 0; nt < 4; ++nt)
        *reinterpret_cast<float2*>(orow + 8 * nt) = make_float2(o[mt][nt][2 * h], o[mt][nt][2 * h + 1]);
      if (warp == 0 && qd == 0)
        *reinterpret_cast<float2*>(p.ml_part + (part * kAttRows + row) * 2) =
            make_float2(m_run[mt][h], l_run[mt][h]);
    }
}

// out[b, token, kvh * G + hg, d] = sum_s w_s O_s[row, d] / sum_s w_s l_s,
// w_s = 2^(m_s - max_s m_s), splits in order.  Grid (rows, KVH, B), 128 threads.
__global__ void __launch_bounds__(kAttD)
    verify_attn_combine_kernel(const float* __restrict__ o_part, const float* __restrict__ ml_part,
                               __nv_bfloat16* __restrict__ out, int H, int KVH, int T, int G,
                               int splits) {
  const int row = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z, d = threadIdx.x;
  pdl_launch_dependents();
  pdl_wait();  // the split partials
  const int64_t base = (static_cast<int64_t>(b) * KVH + kvh) * splits;
  float mx = kMaskedMax;
  for (int s = 0; s < splits; ++s) mx = fmaxf(mx, ml_part[((base + s) * kAttRows + row) * 2]);
  float num = 0.f, den = 0.f;
  for (int s = 0; s < splits; ++s) {
    const float2 ml = *reinterpret_cast<const float2*>(ml_part + ((base + s) * kAttRows + row) * 2);
    const float w = ml.x > 0.5f * kMaskedMax ? exp2f(ml.x - mx) : 0.f;
    num += w * o_part[((base + s) * kAttRows + row) * kAttD + d];
    den += w * ml.y;
  }
  const int hg = row / T, tk = row % T;
  out[((static_cast<int64_t>(b) * T + tk) * H + kvh * G + hg) * kAttD + d] =
      __float2bfloat16_rn(den > 0.f ? num / den : 0.f);
}

// CTAs of verify_attn_kernel resident per SM (shared memory bound: 2 on B200).
int att_ctas_per_sm() {
  static int n = 0;
  if (n == 0) {
    int v = 0;
    if (!set_smem_limit(verify_attn_kernel, kAttSmem) ||
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&v, verify_attn_kernel, kAttThreads, kAttSmem) !=
            cudaSuccess ||
        v < 1)
      v = 1;
    n = v;
  }
  return n;
}

// KV splits per (batch, KV head): minimise waves x (tiles per CTA + 1), the +1
// standing for a CTA's fixed cost (Q load, partial write, its share of the
// combine).  A split count whose last wave is nearly empty costs a whole wave.
int att_splits(int64_t batch, int kv_heads, int len, int num_sms) {
  const int tiles = (len + kAttTile - 1) / kAttTile;
  const int64_t pairs = batch * kv_heads;
  const int64_t slots = static_cast<int64_t>(num_sms) * att_ctas_per_sm();
  int best = 1;
  int64_t best_cost = -1;
  for (int s = 1; s <= tiles; ++s) {
    const int64_t waves = (pairs * s + slots - 1) / slots;
    const int64_t cost = waves * ((tiles + s - 1) / s + 1);
    if (best_cost < 0 || cost < best_cost) {
      best_cost = cost;
      best = s;
    }
  }
  return best;
}

}  // namespace

size_t verify_attention_workspace(int64_t batch, int kv_heads, int len, int num_sms) {
  const int s = att_splits(batch, kv_heads, len, num_sms);
  return static_cast<size_t>(batch) * kv_heads * s * kAttRows * (kAttD + 2) * sizeof(float);
}

int launch_verify_attention(const void* q, const void* k_cache, const void* v_cache, void* out,
                            int64_t batch, int heads, int kv_heads, int t_new, int prefix, int cap,
                            void* workspace, cudaStream_t st, int num_sms) {
  const int len = prefix + t_new;
  const int splits = att_splits(batch, kv_heads, len, num_sms);
  const int tiles = (len + kAttTile - 1) / kAttTile;
  AttParams p;
  p.q = static_cast<const __nv_bfloat16*>(q);
  p.k = static_cast<const __nv_bfloat16*>(k_cache);
  p.v = static_cast<const __nv_bfloat16*>(v_cache);
  p.o_part = static_cast<float*>(workspace);
  p.ml_part = p.o_part + static_cast<int64_t>(batch) * kv_heads * splits * kAttRows * kAttD;
  p.H = heads;
  p.KVH = kv_heads;
  p.T = t_new;
  p.G = heads / kv_heads;
  p.rows = p.G * t_new;
  p.prefix = prefix;
  p.len = len;
  p.cap = cap;
  p.splits = splits;
  p.tiles_per_split = (tiles + splits - 1) / splits;
  p.scale_log2 = 1.4426950408889634f / sqrtf(static_cast<float>(kAttD));
  if (!set_smem_limit(verify_attn_kernel, kAttSmem)) return FITQ_ERR_CUDA;
  cudaError_t e = launch_pdl(verify_attn_kernel, dim3(splits, kv_heads, static_cast<unsigned>(batch)),
                             dim3(kAttThreads), kAttSmem, st, p);
  note_launch();
  if (e != cudaSuccess) return FITQ_ERR_CUDA;
  e = launch_pdl(verify_attn_combine_kernel, dim3(p.rows, kv_heads, static_cast<unsigned>(batch)), dim3(kAttD),
                 0, st, static_cast<const float*>(p.o_part), static_cast<const float*>(p.ml_part),
                 static_cast<__nv_bfloat16*>(out), heads, kv_heads, t_new, p.G, splits);
  note_launch();
  return e == cudaSuccess ? FITQ_OK : FITQ_ERR_CUDA;
}

}  // namespace fitq
