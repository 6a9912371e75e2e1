// Causal grouped-query attention of the training layer, forward and backward.
//
// Replaces the attention inside the Qwen2 decoder layer that FitLLM runs in
// its shard-stationary forward and in the backward's recompute (HF layer via
// fitllm/forward.py:657-701, recompute fitllm/backward.py:222-231):
//   O = softmax(scale . Q K^T + causal mask) V,   scale = 1 / sqrt(head_dim),
// with the H query heads sharing KVH key/value heads (head h reads KV head
// h / (H / KVH)), and its gradients dQ, dK, dV.
//
// Layouts (no transposes around the projections): q, o, dq, do [B, S, H, 128]
// bf16 (the q_proj output / o_proj input as [B, S, H * 128]); k, v, dk, dv
// [B, S, KVH, 128] bf16; lse and delta [B, H, S] fp32.  S % 64 == 0.
//
// Warp-level bf16 tensor-core MMA (mma.sync m16n8k16, fp32 accumulate), the
// FlashAttention-2 organisation:
//   attn_fwd_kernel       grid (S/64, H, B), 4 warps: warp w owns 16 query
//                         rows of a 64-row block, Q fragments in registers;
//                         64-key K/V tiles stream through a cp.async double
//                         buffer (XOR-swizzled 16-byte chunks: conflict-free
//                         ldmatrix); online softmax in base 2, P handed from
//                         the S accumulators to the P.V MMA in registers.
//                         Writes O and lse = m + log2(l) (base-2 units of the
//                         scaled scores).
//   attn_bwd_delta_kernel delta[b, h, s] = sum_d dO . O (fp32).
//   attn_bwd_dkdv_kernel  grid (S/64, KVH, B): warp w owns 16 keys; the CTA
//                         walks every query head of its KV group and every
//                         32-row query step at or after the key block,
//                         recomputing P^T = exp2(K Q^T . c - lse) and
//                         accumulating dV += P^T dO and dK += dS^T Q with
//                         dS = P (dP - delta), dP^T = V dO^T.
//   attn_bwd_dq_kernel    grid (S/64, H, B): warp w owns 16 query rows; 32-key
//                         steps up to the diagonal, dQ += dS K.
// Each output element is one warp's sum in a fixed order (no atomics), so the
// gradients are deterministic.  P and dS are rounded to bf16 for the MMAs,
// as flash-attention kernels do; everything else is fp32.
#include "common.cuh"
#include "kernels.cuh"

namespace fitq {
namespace {

constexpr int kTaD = 128;
constexpr int kTaRow = kTaD * 2;          // 256 B per row of q / k / v
constexpr int kTaThreads = 128;
constexpr int kTaQBlk = 64;               // query rows per forward / dQ CTA
constexpr int kTaKBlk = 64;               // keys per forward tile and per dK/dV CTA
constexpr int kTaBwdQ = 32;               // query rows per dK/dV step
constexpr int kTaBwdK = 32;               // keys per dQ step
constexpr float kTaMasked = -1.0e30f;

// forward: Q 16 KB + two K and two V tiles of 16 KB = 80 KB (two CTAs per SM)
constexpr int kTaFwdSmem = kTaQBlk * kTaRow + 4 * kTaKBlk * kTaRow;
// dK/dV: K, V 32 KB + two (Q, dO) steps of 8 KB each + two (lse, delta) rows
constexpr int kTaDkvStep = 2 * kTaBwdQ * kTaRow + 2 * kTaBwdQ * 4;
constexpr int kTaDkvSmem = 2 * kTaKBlk * kTaRow + 2 * kTaDkvStep;
// dQ: Q, dO 32 KB + two (K, V) steps of 8 KB each
constexpr int kTaDqSmem = 2 * kTaQBlk * kTaRow + 4 * kTaBwdK * kTaRow;

extern __shared__ __align__(128) uint8_t g_ta_smem[];

__device__ __forceinline__ void ta_cp16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void ta_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void ta_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

__device__ __forceinline__ void ta_ldsm(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ta_ldsm_t(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ta_mma(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
      "{%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Byte offset of 16-byte chunk c of row r in a [rows][256 B] tile: chunk XOR
// (r & 7), so the 8 rows of one ldmatrix matrix fall in 8 different banks.
__device__ __forceinline__ uint32_t ta_swz(int r, int c) {
  return static_cast<uint32_t>(r * kTaRow + ((c ^ (r & 7)) << 4));
}

// Copy `rows` rows of 256 B (row r at src + r * ld elements) into a swizzled
// tile; every thread of the CTA takes rows * 16 / 128 chunks.
__device__ __forceinline__ void ta_load_rows(uint32_t dst, const __nv_bfloat16* src, int64_t ld,
                                             int rows) {
  for (int i = threadIdx.x; i < rows * 16; i += kTaThreads) {
    const int r = i >> 4, c = i & 15;
    ta_cp16(dst + ta_swz(r, c), src + static_cast<int64_t>(r) * ld + c * 8);
  }
}

// A fragments (16 rows x 16 columns, k-step ks) of rows r0.. of a swizzled
// tile: matrices (rows 0-7 | 8-15) x (chunk 2 ks | 2 ks + 1) in a0..a3 order.
__device__ __forceinline__ void ta_frag_a(uint32_t tile, int r0, int ks, uint32_t (&a)[4]) {
  const int lane = threadIdx.x & 31, mat = lane >> 3, rr = lane & 7;
  ta_ldsm(tile + ta_swz(r0 + 8 * (mat & 1) + rr, 2 * ks + (mat >> 1)), a);
}
// B fragments of two n8 tiles (rows r0..r0+7 and r0+8..r0+15 of the tile are
// the n index, the 16 columns of k-step ks the k index): {b[0], b[1]} for the
// first n8 tile, {b[2], b[3]} for the second.
__device__ __forceinline__ void ta_frag_b(uint32_t tile, int r0, int ks, uint32_t (&b)[4]) {
  const int lane = threadIdx.x & 31, mat = lane >> 3, rr = lane & 7;
  ta_ldsm(tile + ta_swz(r0 + 8 * (mat >> 1) + rr, 2 * ks + (mat & 1)), b);
}
// B fragments with the tile's rows as the k index (rows r0..r0+15) and its
// columns as the n index: two n8 tiles of columns 8 (2 np) and 8 (2 np + 1).
__device__ __forceinline__ void ta_frag_bt(uint32_t tile, int r0, int np, uint32_t (&b)[4]) {
  const int lane = threadIdx.x & 31, mat = lane >> 3, rr = lane & 7;
  ta_ldsm_t(tile + ta_swz(r0 + 8 * (mat & 1) + rr, 2 * np + (mat >> 1)), b);
}

// A fragment (16 x 16, k = columns 16 kk..16 kk+15) from the fp32 accumulators
// of n8 tiles 2 kk and 2 kk + 1, rounded to bf16.
__device__ __forceinline__ void ta_acc_to_a(const float (&t0)[4], const float (&t1)[4],
                                            uint32_t (&a)[4]) {
  a[0] = pack_bf16x2(t0[0], t0[1]);
  a[1] = pack_bf16x2(t0[2], t0[3]);
  a[2] = pack_bf16x2(t1[0], t1[1]);
  a[3] = pack_bf16x2(t1[2], t1[3]);
}

struct TaParams {
  const __nv_bfloat16* q;
  const __nv_bfloat16* k;
  const __nv_bfloat16* v;
  const __nv_bfloat16* o;
  const __nv_bfloat16* d_o;
  __nv_bfloat16* out;   // forward: O; dQ kernel: dQ
  __nv_bfloat16* dk;
  __nv_bfloat16* dv;
  float* lse;           // [B, H, S]
  float* delta;         // [B, H, S]
  int S, H, KVH, G;
  float scale_log2;     // log2(e) / sqrt(D)
  float scale;          // 1 / sqrt(D)
};

__global__ void __launch_bounds__(kTaThreads, 2) attn_fwd_kernel(const TaParams p) {
  pdl_launch_dependents();
  pdl_wait();  // q, k, v come from the previous kernels
  const int nqb = p.S / kTaQBlk;
  const int qb = nqb - 1 - static_cast<int>(blockIdx.x);  // longest rows first
  const int h = blockIdx.y, b = blockIdx.z, kvh = h / p.G;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, qd = lane & 3;
  const uint32_t s_q = smem_u32(g_ta_smem);
  const uint32_t s_k = s_q + kTaQBlk * kTaRow;  // two K tiles, then two V tiles
  const uint32_t s_v = s_k + 2 * kTaKBlk * kTaRow;
  const int64_t ldq = static_cast<int64_t>(p.H) * kTaD, ldk = static_cast<int64_t>(p.KVH) * kTaD;
  const __nv_bfloat16* kbase = p.k + (static_cast<int64_t>(b) * p.S) * ldk + kvh * kTaD;
  const __nv_bfloat16* vbase = p.v + (static_cast<int64_t>(b) * p.S) * ldk + kvh * kTaD;

  ta_load_rows(s_q, p.q + (static_cast<int64_t>(b) * p.S + qb * kTaQBlk) * ldq + h * kTaD, ldq, kTaQBlk);
  ta_load_rows(s_k, kbase, ldk, kTaKBlk);
  ta_load_rows(s_v, vbase, ldk, kTaKBlk);
  ta_commit();

  uint32_t qa[kTaD / 16][4];
  float o[kTaD / 8][4];
#pragma unroll
  for (int nt = 0; nt < kTaD / 8; ++nt)
#pragma unroll
    for (int e = 0; e < 4; ++e) o[nt][e] = 0.f;
  float m_run[2] = {kTaMasked, kTaMasked}, l_run[2] = {0.f, 0.f};
  const int ntiles = qb + 1;  // causal: key tiles 0..qb
  const int qrow = qb * kTaQBlk + 16 * warp + g;  // query position of e < 2 (e >= 2: + 8)

  for (int t = 0; t < ntiles; ++t) {
    const int buf = t & 1;
    ta_wait_all();
    __syncthreads();  // tile t (and Q) visible; every warp is done with tile t - 1
    if (t == 0) {
#pragma unroll
      for (int ks = 0; ks < kTaD / 16; ++ks) ta_frag_a(s_q, 16 * warp, ks, qa[ks]);
    }
    if (t + 1 < ntiles) {
      const int64_t off = static_cast<int64_t>(t + 1) * kTaKBlk * ldk;
      ta_load_rows(s_k + (buf ^ 1) * kTaKBlk * kTaRow, kbase + off, ldk, kTaKBlk);
      ta_load_rows(s_v + (buf ^ 1) * kTaKBlk * kTaRow, vbase + off, ldk, kTaKBlk);
    }
    ta_commit();
    const uint32_t kt = s_k + buf * kTaKBlk * kTaRow, vt = s_v + buf * kTaKBlk * kTaRow;

    // S = Q K^T: 16 rows x 64 keys (eight n8 tiles)
    float s[kTaKBlk / 8][4];
#pragma unroll
    for (int nt = 0; nt < kTaKBlk / 8; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) s[nt][e] = 0.f;
#pragma unroll
    for (int ks = 0; ks < kTaD / 16; ++ks) {
#pragma unroll
      for (int np = 0; np < kTaKBlk / 16; ++np) {
        uint32_t kf[4];
        ta_frag_b(kt, 16 * np, ks, kf);
        ta_mma(s[2 * np], qa[ks], kf[0], kf[1]);
        ta_mma(s[2 * np + 1], qa[ks], kf[2], kf[3]);
      }
    }

    // scale, causal mask on the diagonal tile, online softmax (base 2)
    const bool diag = t == qb;
    float mx[2] = {kTaMasked, kTaMasked};
#pragma unroll
    for (int nt = 0; nt < kTaKBlk / 8; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int key = t * kTaKBlk + 8 * nt + 2 * qd + (e & 1);
        float v = s[nt][e] * p.scale_log2;
        if (diag && key > qrow + 8 * (e >> 1)) v = kTaMasked;
        s[nt][e] = v;
        mx[e >> 1] = fmaxf(mx[e >> 1], v);
      }
    float alpha[2];
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      mx[hh] = fmaxf(mx[hh], __shfl_xor_sync(0xffffffffu, mx[hh], 1));
      mx[hh] = fmaxf(mx[hh], __shfl_xor_sync(0xffffffffu, mx[hh], 2));
      const float m_new = fmaxf(m_run[hh], mx[hh]);
      alpha[hh] = exp2f(m_run[hh] - m_new);
      m_run[hh] = m_new;
      l_run[hh] *= alpha[hh];
    }
#pragma unroll
    for (int nt = 0; nt < kTaKBlk / 8; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float v = s[nt][e];
        const float pv = v > 0.5f * kTaMasked ? exp2f(v - m_run[e >> 1]) : 0.f;
        s[nt][e] = pv;
        l_run[e >> 1] += pv;
      }
#pragma unroll
    for (int nt = 0; nt < kTaD / 8; ++nt) {
      o[nt][0] *= alpha[0];
      o[nt][1] *= alpha[0];
      o[nt][2] *= alpha[1];
      o[nt][3] *= alpha[1];
    }

    // O += P V
#pragma unroll
    for (int kk = 0; kk < kTaKBlk / 16; ++kk) {
      uint32_t pa[4];
      ta_acc_to_a(s[2 * kk], s[2 * kk + 1], pa);
#pragma unroll
      for (int np = 0; np < kTaD / 16; ++np) {
        uint32_t vf[4];
        ta_frag_bt(vt, 16 * kk, np, vf);
        ta_mma(o[2 * np], pa, vf[0], vf[1]);
        ta_mma(o[2 * np + 1], pa, vf[2], vf[3]);
      }
    }
  }
  ta_wait_all();

#pragma unroll
  for (int hh = 0; hh < 2; ++hh) {
    float l = l_run[hh];
    l += __shfl_xor_sync(0xffffffffu, l, 1);
    l += __shfl_xor_sync(0xffffffffu, l, 2);
    const float inv = 1.0f / l;
    const int row = qrow + 8 * hh;
    __nv_bfloat16* orow = p.out + (static_cast<int64_t>(b) * p.S + row) * ldq + h * kTaD + 2 * qd;
#pragma unroll
    for (int nt = 0; nt < kTaD / 8; ++nt)
      *reinterpret_cast<uint32_t*>(orow + 8 * nt) =
          pack_bf16x2(o[nt][2 * hh] * inv, o[nt][2 * hh + 1] * inv);
    if (qd == 0) p.lse[(static_cast<int64_t>(b) * p.H + h) * p.S + row] = m_run[hh] + log2f(l);
  }
}

// delta[b, h, s] = sum_d dO[b, s, h, d] * O[b, s, h, d]: one warp per row.
__global__ void __launch_bounds__(256) attn_bwd_delta_kernel(const TaParams p, int64_t rows) {
  pdl_launch_dependents();
  pdl_wait();
  const int64_t r = static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (r >= rows) return;
  const uint2 a = __ldg(reinterpret_cast<const uint2*>(p.d_o + r * kTaD) + lane);
  const uint2 c = __ldg(reinterpret_cast<const uint2*>(p.o + r * kTaD) + lane);
  const float2 a0 = unpack_bf16x2(a.x), a1 = unpack_bf16x2(a.y);
  const float2 c0 = unpack_bf16x2(c.x), c1 = unpack_bf16x2(c.y);
  float s = a0.x * c0.x + a0.y * c0.y + a1.x * c1.x + a1.y * c1.y;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if (lane == 0) {
    // r = (b * S + s) * H + h
    const int h = static_cast<int>(r % p.H);
    const int64_t bs = r / p.H;
    const int64_t b = bs / p.S, sq = bs % p.S;
    p.delta[(b * p.H + h) * p.S + sq] = s;
  }
}

__global__ void __launch_bounds__(kTaThreads, 2) attn_bwd_dkdv_kernel(const TaParams p) {
  pdl_launch_dependents();
  pdl_wait();  // q, k, v, dO, lse, delta come from the previous kernels
  const int kb = blockIdx.x;  // key blocks near the start see the most queries: first
  const int kvh = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, qd = lane & 3;
  const uint32_t s_k = smem_u32(g_ta_smem);
  const uint32_t s_v = s_k + kTaKBlk * kTaRow;
  const uint32_t s_step = s_v + kTaKBlk * kTaRow;  // two steps of [Q | dO | lse | delta]
  float* const f_step = reinterpret_cast<float*>(g_ta_smem + 2 * kTaKBlk * kTaRow);
  const int64_t ldq = static_cast<int64_t>(p.H) * kTaD, ldk = static_cast<int64_t>(p.KVH) * kTaD;
  const int key0 = kb * kTaKBlk;

  ta_load_rows(s_k, p.k + (static_cast<int64_t>(b) * p.S + key0) * ldk + kvh * kTaD, ldk, kTaKBlk);
  ta_load_rows(s_v, p.v + (static_cast<int64_t>(b) * p.S + key0) * ldk + kvh * kTaD, ldk, kTaKBlk);

  const int qs0 = key0 / kTaBwdQ;                  // first query step with rows >= key0
  const int per_head = p.S / kTaBwdQ - qs0;
  const int nsteps = p.G * per_head;
  // step u: query head kvh * G + u / per_head, rows 32 (qs0 + u % per_head) ..
  auto load_step = [&](int u, int buf) {
    const int h = kvh * p.G + u / per_head, q0 = (qs0 + u % per_head) * kTaBwdQ;
    const uint32_t base = s_step + buf * kTaDkvStep;
    const int64_t roff = (static_cast<int64_t>(b) * p.S + q0) * ldq + h * kTaD;
    ta_load_rows(base, p.q + roff, ldq, kTaBwdQ);
    ta_load_rows(base + kTaBwdQ * kTaRow, p.d_o + roff, ldq, kTaBwdQ);
    const int64_t loff = (static_cast<int64_t>(b) * p.H + h) * p.S + q0;
    if (threadIdx.x < 16) {  // 32 lse then 32 delta values: 8 chunks each
      const int c = threadIdx.x & 7;
      const float* src = (threadIdx.x < 8 ? p.lse : p.delta) + loff + 4 * c;
      ta_cp16(base + 2 * kTaBwdQ * kTaRow + (threadIdx.x < 8 ? 0 : kTaBwdQ * 4) + 16 * c, src);
    }
  };
  load_step(0, 0);
  ta_commit();

  float dk[kTaD / 8][4], dv[kTaD / 8][4];
#pragma unroll
  for (int nt = 0; nt < kTaD / 8; ++nt)
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      dk[nt][e] = 0.f;
      dv[nt][e] = 0.f;
    }
  const int krow = key0 + 16 * warp + g;  // key of e < 2 (e >= 2: + 8)

  for (int u = 0; u < nsteps; ++u) {
    const int buf = u & 1;
    ta_wait_all();
    __syncthreads();  // step u visible; every warp is done with step u - 1
    if (u + 1 < nsteps) load_step(u + 1, buf ^ 1);
    ta_commit();
    const uint32_t qt = s_step + buf * kTaDkvStep, dot = qt + kTaBwdQ * kTaRow;
    const float* lse_s = f_step + (buf * kTaDkvStep + 2 * kTaBwdQ * kTaRow) / 4;
    const float* del_s = lse_s + kTaBwdQ;
    const int q0 = (qs0 + u % per_head) * kTaBwdQ;

    // S^T = K Q^T and dP^T = V dO^T: 16 keys x 32 queries each
    float st[kTaBwdQ / 8][4], dpt[kTaBwdQ / 8][4];
#pragma unroll
    for (int nt = 0; nt < kTaBwdQ / 8; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        st[nt][e] = 0.f;
        dpt[nt][e] = 0.f;
      }
#pragma unroll
    for (int ks = 0; ks < kTaD / 16; ++ks) {
      uint32_t ka[4], va[4];
      ta_frag_a(s_k, 16 * warp, ks, ka);
      ta_frag_a(s_v, 16 * warp, ks, va);
#pragma unroll
      for (int np = 0; np < kTaBwdQ / 16; ++np) {
        uint32_t qf[4], df[4];
        ta_frag_b(qt, 16 * np, ks, qf);
        ta_frag_b(dot, 16 * np, ks, df);
        ta_mma(st[2 * np], ka, qf[0], qf[1]);
        ta_mma(st[2 * np + 1], ka, qf[2], qf[3]);
        ta_mma(dpt[2 * np], va, df[0], df[1]);
        ta_mma(dpt[2 * np + 1], va, df[2], df[3]);
      }
    }
    // P^T = exp2(S^T c - lse) (0 where key > query), dS^T = P^T (dP^T - delta)
#pragma unroll
    for (int nt = 0; nt < kTaBwdQ / 8; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int qc = 8 * nt + 2 * qd + (e & 1);
        const bool vis = q0 + qc >= krow + 8 * (e >> 1);
        const float pv = vis ? exp2f(st[nt][e] * p.scale_log2 - lse_s[qc]) : 0.f;
        st[nt][e] = pv;
        dpt[nt][e] = pv * (dpt[nt][e] - del_s[qc]);
      }
    // dV += P^T dO, dK += dS^T Q: 16 keys x 128
#pragma unroll
    for (int kk = 0; kk < kTaBwdQ / 16; ++kk) {
      uint32_t pa[4], da[4];
      ta_acc_to_a(st[2 * kk], st[2 * kk + 1], pa);
      ta_acc_to_a(dpt[2 * kk], dpt[2 * kk + 1], da);
#pragma unroll
      for (int np = 0; np < kTaD / 16; ++np) {
        uint32_t of[4], qf[4];
        ta_frag_bt(dot, 16 * kk, np, of);
        ta_frag_bt(qt, 16 * kk, np, qf);
        ta_mma(dv[2 * np], pa, of[0], of[1]);
        ta_mma(dv[2 * np + 1], pa, of[2], of[3]);
        ta_mma(dk[2 * np], da, qf[0], qf[1]);
        ta_mma(dk[2 * np + 1], da, qf[2], qf[3]);
      }
    }
  }
  ta_wait_all();

#pragma unroll
  for (int hh = 0; hh < 2; ++hh) {
    const int64_t off = (static_cast<int64_t>(b) * p.S + krow + 8 * hh) * ldk + kvh * kTaD + 2 * qd;
#pragma unroll
    for (int nt = 0; nt < kTaD / 8; ++nt) {
      *reinterpret_cast<uint32_t*>(p.dk + off + 8 * nt) =
          pack_bf16x2(dk[nt][2 * hh] * p.scale, dk[nt][2 * hh + 1] * p.scale);
      *reinterpret_cast<uint32_t*>(p.dv + off + 8 * nt) = pack_bf16x2(dv[nt][2 * hh], dv[nt][2 * hh + 1]);
    }
  }
}

__global__ void __launch_bounds__(kTaThreads, 2) attn_bwd_dq_kernel(const TaParams p) {
  pdl_launch_dependents();
  pdl_wait();  // q, k, v, dO, lse, delta come from the previous kernels
  const int nqb = p.S / kTaQBlk;
  const int qb = nqb - 1 - static_cast<int>(blockIdx.x);  // longest rows first
  const int h = blockIdx.y, b = blockIdx.z, kvh = h / p.G;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, qd = lane & 3;
  const uint32_t s_q = smem_u32(g_ta_smem);
  const uint32_t s_do = s_q + kTaQBlk * kTaRow;
  const uint32_t s_kv = s_do + kTaQBlk * kTaRow;  // two steps of [K | V]
  const int64_t ldq = static_cast<int64_t>(p.H) * kTaD, ldk = static_cast<int64_t>(p.KVH) * kTaD;
  const int64_t roff = (static_cast<int64_t>(b) * p.S + qb * kTaQBlk) * ldq + h * kTaD;
  const __nv_bfloat16* kbase = p.k + (static_cast<int64_t>(b) * p.S) * ldk + kvh * kTaD;
  const __nv_bfloat16* vbase = p.v + (static_cast<int64_t>(b) * p.S) * ldk + kvh * kTaD;

  ta_load_rows(s_q, p.q + roff, ldq, kTaQBlk);
  ta_load_rows(s_do, p.d_o + roff, ldq, kTaQBlk);
  ta_load_rows(s_kv, kbase, ldk, kTaBwdK);
  ta_load_rows(s_kv + kTaBwdK * kTaRow, vbase, ldk, kTaBwdK);
  ta_commit();

  const int qrow = qb * kTaQBlk + 16 * warp + g;  // query of e < 2 (e >= 2: + 8)
  const int64_t lrow = (static_cast<int64_t>(b) * p.H + h) * p.S + qrow;
  const float lse_r[2] = {__ldg(p.lse + lrow), __ldg(p.lse + lrow + 8)};
  const float del_r[2] = {__ldg(p.delta + lrow), __ldg(p.delta + lrow + 8)};

  uint32_t qa[kTaD / 16][4], da[kTaD / 16][4];
  float dq[kTaD / 8][4];
#pragma unroll
  for (int nt = 0; nt < kTaD / 8; ++nt)
#pragma unroll
    for (int e = 0; e < 4; ++e) dq[nt][e] = 0.f;
  const int nsteps = (qb + 1) * (kTaQBlk / kTaBwdK);  // causal: keys < (qb + 1) * 64

  for (int j = 0; j < nsteps; ++j) {
    const int buf = j & 1;
    ta_wait_all();
    __syncthreads();  // step j (and Q, dO) visible; every warp is done with step j - 1
    if (j == 0) {
#pragma unroll
      for (int ks = 0; ks < kTaD / 16; ++ks) {
        ta_frag_a(s_q, 16 * warp, ks, qa[ks]);
        ta_frag_a(s_do, 16 * warp, ks, da[ks]);
      }
    }
    if (j + 1 < nsteps) {
      const uint32_t nb = s_kv + (buf ^ 1) * 2 * kTaBwdK * kTaRow;
      const int64_t off = static_cast<int64_t>(j + 1) * kTaBwdK * ldk;
      ta_load_rows(nb, kbase + off, ldk, kTaBwdK);
      ta_load_rows(nb + kTaBwdK * kTaRow, vbase + off, ldk, kTaBwdK);
    }
    ta_commit();
    const uint32_t kt = s_kv + buf * 2 * kTaBwdK * kTaRow, vt = kt + kTaBwdK * kTaRow;
    const int key0 = j * kTaBwdK;

    // S = Q K^T and dP = dO V^T: 16 queries x 32 keys
    float s[kTaBwdK / 8][4], dp[kTaBwdK / 8][4];
#pragma unroll
    for (int nt = 0; nt < kTaBwdK / 8; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        s[nt][e] = 0.f;
        dp[nt][e] = 0.f;
      }
#pragma unroll
    for (int ks = 0; ks < kTaD / 16; ++ks) {
#pragma unroll
      for (int np = 0; np < kTaBwdK / 16; ++np) {
        uint32_t kf[4], vf[4];
        ta_frag_b(kt, 16 * np, ks, kf);
        ta_frag_b(vt, 16 * np, ks, vf);
        ta_mma(s[2 * np], qa[ks], kf[0], kf[1]);
        ta_mma(s[2 * np + 1], qa[ks], kf[2], kf[3]);
        ta_mma(dp[2 * np], da[ks], vf[0], vf[1]);
        ta_mma(dp[2 * np + 1], da[ks], vf[2], vf[3]);
      }
    }
    // P = exp2(S c - lse) (0 where key > query), dS = P (dP - delta)
#pragma unroll
    for (int nt = 0; nt < kTaBwdK / 8; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int key = key0 + 8 * nt + 2 * qd + (e & 1);
        const bool vis = key <= qrow + 8 * (e >> 1);
        const float pv = vis ? exp2f(s[nt][e] * p.scale_log2 - lse_r[e >> 1]) : 0.f;
        dp[nt][e] = pv * (dp[nt][e] - del_r[e >> 1]);
      }
    // dQ += dS K: 16 queries x 128
#pragma unroll
    for (int kk = 0; kk < kTaBwdK / 16; ++kk) {
      uint32_t dsa[4];
      ta_acc_to_a(dp[2 * kk], dp[2 * kk + 1], dsa);
#pragma unroll
      for (int np = 0; np < kTaD / 16; ++np) {
        uint32_t kf[4];
        ta_frag_bt(kt, 16 * kk, np, kf);
        ta_mma(dq[2 * np], dsa, kf[0], kf[1]);
        ta_mma(dq[2 * np + 1], dsa, kf[2], kf[3]);
      }
    }
  }
  ta_wait_all();

#pragma unroll
  for (int hh = 0; hh < 2; ++hh) {
    __nv_bfloat16* row =
        p.out + (static_cast<int64_t>(b) * p.S + qrow + 8 * hh) * ldq + h * kTaD + 2 * qd;
#pragma unroll
    for (int nt = 0; nt < kTaD / 8; ++nt)
      *reinterpret_cast<uint32_t*>(row + 8 * nt) =
          pack_bf16x2(dq[nt][2 * hh] * p.scale, dq[nt][2 * hh + 1] * p.scale);
  }
}

TaParams ta_params(int64_t batch, int64_t seq, int heads, int kv_heads) {
  TaParams p{};
  p.S = static_cast<int>(seq);
  p.H = heads;
  p.KVH = kv_heads;
  p.G = heads / kv_heads;
  p.scale = 1.0f / sqrtf(static_cast<float>(kTaD));
  p.scale_log2 = 1.4426950408889634f * p.scale;
  (void)batch;
  return p;
}

}  // namespace

int launch_train_attn_fwd(const void* q, const void* k, const void* v, void* out, float* lse,
                          int64_t batch, int64_t seq, int heads, int kv_heads, cudaStream_t st) {
  TaParams p = ta_params(batch, seq, heads, kv_heads);
  p.q = static_cast<const __nv_bfloat16*>(q);
  p.k = static_cast<const __nv_bfloat16*>(k);
  p.v = static_cast<const __nv_bfloat16*>(v);
  p.out = static_cast<__nv_bfloat16*>(out);
  p.lse = lse;
  if (!set_smem_limit(attn_fwd_kernel, kTaFwdSmem)) return FITQ_ERR_CUDA;
  const cudaError_t e =
      launch_pdl(attn_fwd_kernel, dim3(static_cast<unsigned>(seq / kTaQBlk), heads, static_cast<unsigned>(batch)),
                 dim3(kTaThreads), kTaFwdSmem, st, p);
  note_launch();
  return e == cudaSuccess ? FITQ_OK : FITQ_ERR_CUDA;
}

int launch_train_attn_bwd(const void* q, const void* k, const void* v, const void* o,
                          const void* d_o, const float* lse, void* dq, void* dk, void* dv,
                          float* delta, int64_t batch, int64_t seq, int heads, int kv_heads,
                          cudaStream_t st) {
  TaParams p = ta_params(batch, seq, heads, kv_heads);
  p.q = static_cast<const __nv_bfloat16*>(q);
  p.k = static_cast<const __nv_bfloat16*>(k);
  p.v = static_cast<const __nv_bfloat16*>(v);
  p.o = static_cast<const __nv_bfloat16*>(o);
  p.d_o = static_cast<const __nv_bfloat16*>(d_o);
  p.out = static_cast<__nv_bfloat16*>(dq);
  p.dk = static_cast<__nv_bfloat16*>(dk);
  p.dv = static_cast<__nv_bfloat16*>(dv);
  p.lse = const_cast<float*>(lse);
  p.delta = delta;
  if (!set_smem_limit(attn_bwd_dkdv_kernel, kTaDkvSmem) || !set_smem_limit(attn_bwd_dq_kernel, kTaDqSmem))
    return FITQ_ERR_CUDA;
  const int64_t rows = batch * seq * heads;
  cudaError_t e = launch_pdl(attn_bwd_delta_kernel, dim3(static_cast<unsigned>((rows + 7) / 8)), dim3(256),
                             0, st, p, rows);
  note_launch();
  if (e != cudaSuccess) return FITQ_ERR_CUDA;
  e = launch_pdl(attn_bwd_dkdv_kernel,
                 dim3(static_cast<unsigned>(seq / kTaKBlk), kv_heads, static_cast<unsigned>(batch)),
                 dim3(kTaThreads), kTaDkvSmem, st, p);
  note_launch();
  if (e != cudaSuccess) return FITQ_ERR_CUDA;
  e = launch_pdl(attn_bwd_dq_kernel,
                 dim3(static_cast<unsigned>(seq / kTaQBlk), heads, static_cast<unsigned>(batch)),
                 dim3(kTaThreads), kTaDqSmem, st, p);
  note_launch();
  return e == cudaSuccess ? FITQ_OK : FITQ_ERR_CUDA;
}

}  // namespace fitq
