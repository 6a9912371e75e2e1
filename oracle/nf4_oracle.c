/*
 * CPU oracle for the NF4 QLoRA hot path -- TEST INFRASTRUCTURE ONLY.
 *
 * This file restates, in plain C, the arithmetic that FitLLM's QLoRA layers get
 * from bitsandbytes (4-bit NormalFloat, blocksize 64, double-quantised absmax).
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may load
 * it, and only as the checker; the product path never links or calls it.
 *
 * Parity status: the NF4 dequant op order is pinned by the call sites that the
 * reference relies on (fitllm/forward.py:76-109 restores QuantState from the flat
 * keys; the nested-absmax reconstruction is blockwise dequant then "+= offset",
 * two separately rounded fp32 ops, as written out in the installed
 * vllm/model_executor/model_loader/bitsandbytes_loader.py:600-601).  bitsandbytes
 * itself is not installed anywhere reachable, so no bnb-produced golden vector
 * exists: the quantiser (absmax, nearest level, double quant) is this project's
 * own restatement of the published method and is parity-UNPINNED against bnb.
 *
 * Data layout (bitsandbytes Params4bit, fitllm/forward.py:95-109 key set):
 *   packed[i]      uint8, flat row-major W[N,K]; element 2i in the HIGH nibble,
 *                  element 2i+1 in the LOW nibble.
 *   absmax_code[b] uint8, one per 64 consecutive flat elements.
 *   nested_absmax  fp32, one per 256 consecutive absmax codes.
 *   quant_map      fp32[16]  (NF4 levels), nested_quant_map fp32[256]
 *                  (signed 8-bit dynamic map), offset fp32.
 *
 * Build: see oracle/Makefile (gcc -O2 -ffp-contract=off: no FMA contraction, so
 * every product and sum below is a single correctly rounded fp32 operation).
 */
#include <stdint.h>
#include <string.h>
#include <math.h>

#define NF4_BLOCK 64
#define DQ_BLOCK 256
#define OFFSET_CHUNK 4096

/* ---- scalar conversions (round to nearest even) ------------------------- */

static inline uint32_t f32_bits(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float bits_f32(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

uint16_t oracle_f32_to_bf16(float f) {
    uint32_t u = f32_bits(f);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x0040u); /* quiet NaN */
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

float oracle_bf16_to_f32(uint16_t h) { return bits_f32(((uint32_t)h) << 16); }

uint16_t oracle_f32_to_f16(float f) {
    uint32_t u = f32_bits(f);
    uint32_t sign = (u >> 16) & 0x8000u;
    uint32_t a = u & 0x7fffffffu;
    if (a > 0x7f800000u) return (uint16_t)(sign | 0x7e00u);            /* NaN */
    if (a >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u);           /* rounds to inf */
    if (a < 0x38800000u) {                                             /* f16 subnormal or zero */
        /* value = a_float; f16 subnormal unit = 2^-24.  Scale exactly and round. */
        uint32_t e = a >> 23;
        if (e < 102) return (uint16_t)sign;                            /* < 2^-25: rounds to 0 */
        uint32_t m = (a & 0x7fffffu) | 0x800000u;                      /* 24-bit significand */
        uint32_t shift = 126 - e;                                      /* 14..24 */
        uint32_t q = m >> shift;
        uint32_t rem = m & ((1u << shift) - 1u);
        uint32_t half = 1u << (shift - 1);
        if (rem > half || (rem == half && (q & 1u))) q++;
        return (uint16_t)(sign | q);
    }
    /* normal: rebias exponent 127 -> 15 and round 23 -> 10 mantissa bits */
    uint32_t r = a - 0x38000000u;                                      /* exponent rebias */
    r += 0xfffu + ((r >> 13) & 1u);
    return (uint16_t)(sign | (r >> 13));
}

/* ---- nearest-level search ------------------------------------------------
 * Levels are sorted ascending.  Threshold t_j = 0.5f * (lv[j] + lv[j+1]) in
 * fp32; the code is the number of thresholds strictly below x, i.e. ties go to
 * the lower level.  This is the decision rule of bitsandbytes' NF4 comparison
 * tree (midpoints, "x > t" selects the upper branch), stated for any sorted table.
 */
static void make_thresholds(const float* lv, int n, float* t) {
    for (int j = 0; j + 1 < n; ++j) t[j] = 0.5f * (lv[j] + lv[j + 1]);
}

static inline int count_below(const float* t, int nt, float x) {
    int lo = 0, hi = nt;           /* first index with !(t[idx] < x) */
    while (lo < hi) {
        int mid = (lo + hi) >> 1;
        if (t[mid] < x) lo = mid + 1; else hi = mid;
    }
    return lo;
}

/* ---- NF4 blockwise quantisation (first level) ---------------------------
 * For each 64-element block: absmax = max |w|; x = w * (1/absmax) (IEEE
 * reciprocal, then one rounded multiply); code = nearest NF4 level.
 * absmax == 0 uses a reciprocal of 0, so every element maps to level 0.0.
 * n must be a multiple of 64.
 */
void oracle_nf4_quantize(const float* w, int64_t n, const float* qmap16,
                         uint8_t* packed, float* absmax) {
    float t[15];
    make_thresholds(qmap16, 16, t);
    int64_t nb = n / NF4_BLOCK;
    for (int64_t b = 0; b < nb; ++b) {
        const float* wb = w + b * NF4_BLOCK;
        float am = 0.0f;
        for (int i = 0; i < NF4_BLOCK; ++i) { float a = fabsf(wb[i]); if (a > am) am = a; }
        absmax[b] = am;
        float inv = am > 0.0f ? 1.0f / am : 0.0f;
        for (int i = 0; i < NF4_BLOCK; i += 2) {
            int c0 = count_below(t, 15, wb[i] * inv);
            int c1 = count_below(t, 15, wb[i + 1] * inv);
            packed[(b * NF4_BLOCK + i) >> 1] = (uint8_t)((c0 << 4) | c1);
        }
    }
}

/* ---- deterministic offset (mean of absmax) ------------------------------
 * sum in double over consecutive chunks of 4096 values (in index order), then
 * the chunk sums in order, then one division and one rounding to fp32.  The
 * device quantiser uses the same association so both produce the same offset.
 */
float oracle_absmax_offset(const float* absmax, int64_t nb) {
    double total = 0.0;
    for (int64_t c = 0; c < nb; c += OFFSET_CHUNK) {
        double part = 0.0;
        int64_t e = c + OFFSET_CHUNK < nb ? c + OFFSET_CHUNK : nb;
        for (int64_t i = c; i < e; ++i) part += (double)absmax[i];
        total += part;
    }
    return (float)(total / (double)nb);
}

/* ---- double quantisation of the absmax vector ---------------------------
 * centred = absmax - offset (fp32); per 256 consecutive values: nabs = max
 * |centred|; x = centred * (1/nabs); code = nearest entry of the 256-entry
 * signed dynamic map (sorted ascending).
 */
void oracle_dq_quantize(const float* absmax, int64_t nb, const float* nqmap256,
                        float offset, uint8_t* codes, float* nested_absmax) {
    float t[255];
    make_thresholds(nqmap256, 256, t);
    int64_t nn = (nb + DQ_BLOCK - 1) / DQ_BLOCK;
    for (int64_t g = 0; g < nn; ++g) {
        int64_t s = g * DQ_BLOCK, e = s + DQ_BLOCK < nb ? s + DQ_BLOCK : nb;
        float m = 0.0f;
        for (int64_t i = s; i < e; ++i) { float a = fabsf(absmax[i] - offset); if (a > m) m = a; }
        nested_absmax[g] = m;
        float inv = m > 0.0f ? 1.0f / m : 0.0f;
        for (int64_t i = s; i < e; ++i) {
            float c = absmax[i] - offset;
            codes[i] = (uint8_t)count_below(t, 255, c * inv);
        }
    }
}

/* ---- dequantisation -----------------------------------------------------
 * absmax_b = fl( fl(nested_quant_map[code_b] * nested_absmax[b/256]) + offset )
 * w        = fl( quant_map[nibble] * absmax_b ), then rounded to the output type.
 * out_kind: 0 = bf16 (uint16 bits), 1 = fp16 (uint16 bits), 2 = fp32.
 */
void oracle_absmax_decode(const uint8_t* codes, const float* nested_absmax,
                          const float* nqmap256, float offset, int64_t nb, float* out) {
    for (int64_t b = 0; b < nb; ++b) {
        float p = nqmap256[codes[b]] * nested_absmax[b / DQ_BLOCK];
        out[b] = p + offset;
    }
}

void oracle_nf4_dequant(const uint8_t* packed, const uint8_t* codes,
                        const float* nested_absmax, const float* qmap16,
                        const float* nqmap256, float offset, int64_t n,
                        int out_kind, void* out) {
    int64_t nb = n / NF4_BLOCK;
    for (int64_t b = 0; b < nb; ++b) {
        float p = nqmap256[codes[b]] * nested_absmax[b / DQ_BLOCK];
        float am = p + offset;
        for (int i = 0; i < NF4_BLOCK; ++i) {
            int64_t e = b * NF4_BLOCK + i;
            uint8_t byte = packed[e >> 1];
            int nib = (e & 1) ? (byte & 0x0f) : (byte >> 4);
            float v = qmap16[nib] * am;
            if (out_kind == 0) ((uint16_t*)out)[e] = oracle_f32_to_bf16(v);
            else if (out_kind == 1) ((uint16_t*)out)[e] = oracle_f32_to_f16(v);
            else ((float*)out)[e] = v;
        }
    }
}

/* Single-level variant (nested == False): absmax already fp32. */
void oracle_nf4_dequant_plain(const uint8_t* packed, const float* absmax,
                              const float* qmap16, int64_t n, int out_kind, void* out) {
    int64_t nb = n / NF4_BLOCK;
    for (int64_t b = 0; b < nb; ++b) {
        float am = absmax[b];
        for (int i = 0; i < NF4_BLOCK; ++i) {
            int64_t e = b * NF4_BLOCK + i;
            uint8_t byte = packed[e >> 1];
            int nib = (e & 1) ? (byte & 0x0f) : (byte >> 4);
            float v = qmap16[nib] * am;
            if (out_kind == 0) ((uint16_t*)out)[e] = oracle_f32_to_bf16(v);
            else if (out_kind == 1) ((uint16_t*)out)[e] = oracle_f32_to_f16(v);
            else ((float*)out)[e] = v;
        }
    }
}
