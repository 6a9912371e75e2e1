// Bit-exact NF4 block decode into a tcgen05 shared-memory operand, shared by
// the fused NF4 GEMMs.
//
// One thread decodes one 64-weight block (32 packed bytes) of one W row:
//   table:  entry i = bf16_rn(fl(quant_map[i] * absmax)) for the 16 codes
//           (pair-wise fp32 products, mul.rn.f32x2), held as two byte planes
//           of four registers (L: low bytes, H: high bytes; entries 4j..4j+3
//           in register j);
//   lookup: two prmt per plane pick the bytes of four codes (three selector
//           bits) and a mask from the fourth bit selects the upper eight
//           entries; two more prmt interleave the planes into bf16 pairs;
//   store:  the 128-byte operand row, 16-byte chunk c at (c ^ row % 8) of the
//           128-byte swizzle pattern (the layout TMA's 128-byte swizzle gives,
//           which the MMA's shared-memory descriptors describe).
#pragma once
#include "common.cuh"

namespace fitq {

__device__ __forceinline__ uint32_t prmt_b32(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
}

// Generic-proxy shared-memory writes become visible to the tensor core (async proxy).
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Shared-memory descriptor of an MN-major, 128-byte-swizzled operand with
// `lbo` bytes between 64-element MN atoms and `sbo` bytes between 8-row K groups.
__device__ __forceinline__ uint64_t umma_smem_desc_sw128_mn(uint32_t saddr, uint32_t lbo,
                                                           uint32_t sbo) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1u) << 46;
  d |= static_cast<uint64_t>(2u) << 61;
  return d;
}

// Packed pair of fp32 values and the pair-wise IEEE product (mul.rn.f32x2:
// each lane rounds like __fmul_rn).
__device__ __forceinline__ uint64_t f32x2(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ uint64_t mul_rn_f32x2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint32_t bf16x2_of(uint64_t v) {
  float lo, hi;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
  return pack_bf16x2(lo, hi);
}

// quant_map as eight packed pairs {qm[2j], qm[2j+1]}.
__device__ __forceinline__ void nf4_load_qm_pairs(const float* qm, uint64_t (&qm2)[8]) {
#pragma unroll
  for (int j = 0; j < 8; ++j) qm2[j] = f32x2(__ldg(qm + 2 * j), __ldg(qm + 2 * j + 1));
}

// The block's table as byte planes.
__device__ __forceinline__ void nf4_block_table(const uint64_t (&qm2)[8], float am, uint32_t (&L)[4],
                                                uint32_t (&H)[4]) {
  const uint64_t am2 = f32x2(am, am);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t e01 = bf16x2_of(mul_rn_f32x2(qm2[2 * i], am2));
    const uint32_t e23 = bf16x2_of(mul_rn_f32x2(qm2[2 * i + 1], am2));
    L[i] = prmt_b32(e01, e23, 0x6420u);
    H[i] = prmt_b32(e01, e23, 0x7531u);
  }
}

// Four weights from selector s (nibbles e1, e0, e3, e2 of two packed bytes
// (e0 << 4 | e1), (e2 << 4 | e3), bit 3 cleared) and mask m (0xFF in the
// output bytes whose nibble has bit 3 set).
__device__ __forceinline__ void nf4_lookup4(uint32_t s, uint32_t m, const uint32_t (&L)[4],
                                            const uint32_t (&H)[4], uint32_t& w01, uint32_t& w23) {
  const uint32_t lo = (prmt_b32(L[0], L[1], s) & ~m) | (prmt_b32(L[2], L[3], s) & m);
  const uint32_t hi = (prmt_b32(H[0], H[1], s) & ~m) | (prmt_b32(H[2], H[3], s) & m);
  w01 = prmt_b32(lo, hi, 0x4051u);  // e0 | e1 << 16
  w23 = prmt_b32(lo, hi, 0x6273u);  // e2 | e3 << 16
}

// Eight weights (one packed 32-bit word, 16 output bytes): selectors and
// masks of both halves computed once per word.
__device__ __forceinline__ uint4 nf4_decode_word(uint32_t w, const uint32_t (&L)[4],
                                                 const uint32_t (&H)[4]) {
  const uint32_t s = w & 0x77777777u;
  const uint32_t t = (w >> 1) & 0x44444444u;
  const uint32_t m0 = prmt_b32(0u, 0xFFFFFFFFu, t);
  const uint32_t m1 = prmt_b32(0u, 0xFFFFFFFFu, t >> 16);
  uint4 o;
  nf4_lookup4(s, m0, L, H, o.x, o.y);
  nf4_lookup4(s >> 16, m1, L, H, o.z, o.w);
  return o;
}

// Decode the 32 packed bytes at src (16-byte aligned shared memory) into the
// 128-byte swizzled operand row at dst (swz = row % 8).
__device__ __forceinline__ void nf4_decode_row(const uint8_t* src, uint8_t* dst, uint32_t swz,
                                               const uint64_t (&qm2)[8], float am) {
  const uint4 q0 = *reinterpret_cast<const uint4*>(src);
  const uint4 q1 = *reinterpret_cast<const uint4*>(src + 16);
  uint32_t L[4], H[4];
  nf4_block_table(qm2, am, L, H);
  const uint32_t words[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
#pragma unroll
  for (int c = 0; c < 8; ++c)
    *reinterpret_cast<uint4*>(dst + ((static_cast<uint32_t>(c) ^ swz) << 4)) =
        nf4_decode_word(words[c], L, H);
}

}  // namespace fitq
