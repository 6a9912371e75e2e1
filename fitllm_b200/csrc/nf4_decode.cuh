// Bit-exact NF4 block decode into a tcgen05 shared-memory operand, shared by
// the fused NF4 GEMMs.
//
// One thread decodes one 64-weight block (32 packed bytes) of one W row:
//   table:  entry i = bf16_rn(fl(quant_map[i] * absmax)) for the 16 codes,
//           held as two byte planes of four registers (L: low bytes, H: high
//           bytes; entries 4j..4j+3 in register j);
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

// The block's table as byte planes.
__device__ __forceinline__ void nf4_block_table(const float (&qm)[16], float am, uint32_t (&L)[4],
                                                uint32_t (&H)[4]) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t e01 = pack_bf16x2(__fmul_rn(qm[4 * i], am), __fmul_rn(qm[4 * i + 1], am));
    const uint32_t e23 = pack_bf16x2(__fmul_rn(qm[4 * i + 2], am), __fmul_rn(qm[4 * i + 3], am));
    L[i] = prmt_b32(e01, e23, 0x6420u);
    H[i] = prmt_b32(e01, e23, 0x7531u);
  }
}

// Four weights from the 16-bit half h of a packed word: for packed bytes
// (e0 << 4 | e1), (e2 << 4 | e3) the nibbles of h are e1, e0, e3, e2.
__device__ __forceinline__ void nf4_lookup4(uint32_t h, const uint32_t (&L)[4],
                                            const uint32_t (&H)[4], uint32_t& w01, uint32_t& w23) {
  const uint32_t s = h & 0x7777u;
  const uint32_t m = prmt_b32(0u, 0xFFFFFFFFu, (h >> 1) & 0x4444u);  // 0xFF where bit 3 set
  const uint32_t lo = (prmt_b32(L[0], L[1], s) & ~m) | (prmt_b32(L[2], L[3], s) & m);
  const uint32_t hi = (prmt_b32(H[0], H[1], s) & ~m) | (prmt_b32(H[2], H[3], s) & m);
  w01 = prmt_b32(lo, hi, 0x4051u);  // e0 | e1 << 16
  w23 = prmt_b32(lo, hi, 0x6273u);  // e2 | e3 << 16
}

// Decode the 32 packed bytes at src (16-byte aligned shared memory) into the
// 128-byte swizzled operand row at dst (swz = row % 8).
__device__ __forceinline__ void nf4_decode_row(const uint8_t* src, uint8_t* dst, uint32_t swz,
                                               const float (&qm)[16], float am) {
  const uint4 q0 = *reinterpret_cast<const uint4*>(src);
  const uint4 q1 = *reinterpret_cast<const uint4*>(src + 16);
  uint32_t L[4], H[4];
  nf4_block_table(qm, am, L, H);
  const uint32_t words[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    uint4 o;
    nf4_lookup4(words[c], L, H, o.x, o.y);
    nf4_lookup4(words[c] >> 16, L, H, o.z, o.w);
    *reinterpret_cast<uint4*>(dst + ((static_cast<uint32_t>(c) ^ swz) << 4)) = o;
  }
}

}  // namespace fitq
