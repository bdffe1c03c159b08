// moe_format.h -- formats, shapes and bit-exact helpers shared by the CUDA kernels and the CPU oracle.
//
// Everything here is plain C++ that compiles for the host and, under nvcc, for the device
// (LK_HD = __host__ __device__), so the oracle and the kernels evaluate the same operations in the
// same order:
//   * IQ2_XXS block layout (GGUF / ggml format, 66 bytes per 256 weights),
//   * the seeded counter-based IQ2_XXS weight generator (identical bytes on CPU and GPU),
//   * software fp32 <-> fp16 conversion (round to nearest even),
//   * lk_expf: an exp restated from its mathematics (Cody-Waite reduction + Taylor polynomial),
//     used for the router sigmoid and SwiGLU on both sides,
//   * q8-per-32 activation quantisation of one 32-element group.
#pragma once
#include <stdint.h>
#include <string.h>
#include <math.h>

#if defined(__CUDACC__)
#define LK_HD __host__ __device__ __forceinline__
#else
#define LK_HD inline
#endif

namespace lk {

// ---- DeepSeek-R1 MoE layer shapes (the reference's fused_layer.cu:18 constants E, HSH, QK)
constexpr int HIDDEN = 7168;        // E: model width, K of gate/up, rows of down
constexpr int MOE_INTER = 2048;     // HSH: expert intermediate width, rows of gate/up, K of down
constexpr int N_EXPERTS = 256;      // routed experts per layer
constexpr int MAX_TOPK = 8;         // router keeps up to 8 (the engine's KE <= 8)
constexpr int QK = 256;             // weights per IQ2_XXS superblock
constexpr int BLK_IQ2 = 66;         // bytes per IQ2_XXS superblock: fp16 d + 8 x (4 grid idx, u32 aux)

// ---- IQ2_XXS sizes (ggml_row_size(IQ2_XXS, K) = K/256*66)
LK_HD constexpr size_t iq2_row_bytes(int K) { return (size_t)(K / QK) * BLK_IQ2; }
LK_HD constexpr size_t iq2_matrix_bytes(int rows, int K) { return (size_t)rows * iq2_row_bytes(K); }
// one expert's gate (or up) = [MOE_INTER rows][HIDDEN]; down = [HIDDEN rows][MOE_INTER]; both 3 784 704 B
constexpr size_t EXPERT_GU_BYTES = (size_t)MOE_INTER * (HIDDEN / QK) * BLK_IQ2;
constexpr size_t EXPERT_DOWN_BYTES = (size_t)HIDDEN * (MOE_INTER / QK) * BLK_IQ2;

// ---- format ids, numerically equal to the reference's FL_Q6K / FL_Q5K / FL_IQ2 / FL_Q2K / FL_Q3K
//      (src/fused_layer.h:11)
enum { FMT_Q6K = 1, FMT_Q5K = 3, FMT_IQ2 = 4, FMT_Q2K = 5, FMT_Q3K = 6 };

// ---- the K-quant down formats (GGUF / ggml block layouts; the reference's BLK_Q2 / BLK_Q3,
//  fused_layer.cu:19).  256 weights per block; weight i = 128n + 32j + 16s + l (n < 2, j < 4, s < 2,
//  l < 16) sits in byte 32n + 16s + l of qs at bits 2j..2j+1, and its 16-weight sub-block has scale
//  index 8n + 2j + s.
//   Q2_K (84 B): scales[16] (bits 0-3 scale, 4-7 min), qs[64], fp16 d, fp16 dmin;
//                w = d*(sc & 15)*q - dmin*(sc >> 4), q in 0..3
//   Q3_K (110 B): hmask[32], qs[64], scales[12] (16 x 6 bits, stored + 32), fp16 d;
//                w = d*(scale - 32)*(q - (hmask[16s + l] bit (4n + j) ? 0 : 4)), q in 0..3
constexpr int BLK_Q2K = 84;
constexpr int BLK_Q3K = 110;
constexpr int Q2K_QS = 16, Q2K_D = 80, Q2K_DMIN = 82;
constexpr int Q3K_QS = 32, Q3K_SC = 96, Q3K_D = 108;
// ---- the shared expert's formats in the real model (the reference's BLK_Q5 / BLK_Q6; W->sh_gate / sh_up
//  Q5_K, sh_down Q6_K, src/fused_layer.h:14).  256 weights per block.
//   Q5_K (176 B): fp16 d, fp16 dmin, scales[12] (8 x (6-bit scale, 6-bit min)), qh[32], qs[128].  Weight
//                i = 64j + 32u + l (j < 4, u < 2, l < 32): q = ((qs[32j + l] >> 4u) & 15) | (qh[l] bit
//                2j + u) << 4, in 0..31; its 32-weight sub-block is 2j + u with (scale, min) from
//                q5k_scale_min; w = d*scale*q - dmin*min.
//   Q6_K (210 B): ql[128], qh[64], scales[16] (int8), fp16 d.  Weight i = 128n + 32c + l (n < 2, c < 4,
//                l < 32): q = ((ql[64n + 32(c & 1) + l] >> 4(c >> 1)) & 15) | ((qh[32n + l] >> 2c) & 3) << 4,
//                value q - 32; its 16-weight sub-block is i / 16; w = d*scales[i / 16]*(q - 32).
constexpr int BLK_Q5K = 176;
constexpr int BLK_Q6K = 210;
constexpr int Q5K_SC = 4, Q5K_QH = 16, Q5K_QS = 48;
constexpr int Q6K_QH = 128, Q6K_SC = 192, Q6K_D = 208;
LK_HD constexpr int fmt_block_bytes(int fmt) {
    return fmt == FMT_Q2K ? BLK_Q2K : fmt == FMT_Q3K ? BLK_Q3K : fmt == FMT_Q5K ? BLK_Q5K : fmt == FMT_Q6K ? BLK_Q6K : BLK_IQ2;
}
// one expert's down matrix [HIDDEN rows][MOE_INTER] in format fmt: 3 784 704 / 4 816 896 / 6 307 840 B
LK_HD constexpr size_t down_matrix_bytes(int fmt) { return (size_t)HIDDEN * (MOE_INTER / QK) * fmt_block_bytes(fmt); }
// one gate (or up) matrix [MOE_INTER rows][HIDDEN] in format fmt: 3 784 704 (IQ2_XXS) / 10 092 544 (Q5_K) B
LK_HD constexpr size_t gu_matrix_bytes(int fmt) { return (size_t)MOE_INTER * (HIDDEN / QK) * fmt_block_bytes(fmt); }

// Q3_K's 6-bit scale i (0..15) from the 12 packed bytes: low 4 bits in byte i (i < 8) or the high
// nibble of byte i - 8, high 2 bits at bits 2*(i/4) of byte 8 + i%4 (ggml dequantize_row_q3_K's
// kmask unpacking; the reference's q3_scales, fused_layer.cu:34-37).  Returns scale - 32.
LK_HD int q3k_scale(const uint8_t* sc, int i) {
    const int lo = i < 8 ? (sc[i] & 15) : (sc[i - 8] >> 4);
    const int hi = (sc[8 + (i & 3)] >> (2 * (i >> 2))) & 3;
    return (lo | (hi << 4)) - 32;
}

// Q5_K's (scale, min) of 32-weight sub-block j (0..7) from the 12 packed bytes (ggml get_scale_min_k4; the
// reference's scale_min, fused_layer.cu:25-26): j < 4: low 6 bits of bytes j and j + 4; else the nibbles
// of byte j + 4 with the top 2 bits of bytes j - 4 (scale) and j (min) as bits 4-5.
LK_HD void q5k_scale_min(const uint8_t* sc, int j, int& scale, int& mn) {
    if (j < 4) { scale = sc[j] & 63; mn = sc[j + 4] & 63; }
    else { scale = (sc[j + 4] & 15) | ((sc[j - 4] >> 6) << 4); mn = (sc[j + 4] >> 4) | ((sc[j] >> 6) << 4); }
}

// ---- fp16 <-> fp32 in software (IEEE binary16, round to nearest even), identical on host and device
LK_HD uint32_t f32_bits(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
LK_HD float bits_f32(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

LK_HD float half_to_float(uint16_t h) {
    const uint32_t s = (uint32_t)(h & 0x8000u) << 16, e = (h >> 10) & 0x1Fu, m = h & 0x3FFu;
    if (e == 0) {                                   // zero / subnormal: m * 2^-24, exact in fp32
        const float v = (float)m * 5.9604644775390625e-08f;
        return s ? -v : v;
    }
    if (e == 31) return bits_f32(s | 0x7F800000u | (m << 13));
    return bits_f32(s | ((e + 112u) << 23) | (m << 13));
}

LK_HD uint16_t float_to_half_rne(float f) {
    const uint32_t x = f32_bits(f), s = (x >> 16) & 0x8000u;
    const uint32_t ax = x & 0x7FFFFFFFu;
    if (ax >= 0x7F800000u) return (uint16_t)(s | 0x7C00u | (ax > 0x7F800000u ? 0x200u : 0u));
    if (ax >= 0x477FF000u) return (uint16_t)(s | 0x7C00u);          // rounds to >= 65520: inf
    if (ax < 0x38800000u) {                                         // result subnormal (or zero)
        if (ax < 0x33000000u) return (uint16_t)s;                   // < 2^-25: rounds to 0
        const uint32_t e = ax >> 23, m = (ax & 0x7FFFFFu) | 0x800000u;
        const uint32_t shift = 126u - e;                            // 14..24 (value = m * 2^(e-150), unit 2^-24)
        uint32_t q = m >> shift; const uint32_t rem = m & ((1u << shift) - 1u), half = 1u << (shift - 1u);
        if (rem > half || (rem == half && (q & 1u))) ++q;
        return (uint16_t)(s | q);
    }
    uint32_t q = ((ax >> 13) - (112u << 10));                       // rebias exponent, keep 10 mantissa bits
    const uint32_t rem = ax & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (q & 1u))) ++q;        // carry into the exponent is correct
    return (uint16_t)(s | q);
}

// ---- exp(x) for fp32, restated from its mathematics, bit-identical on CPU and GPU.
//  n = rint(x / ln2); r = x - n*ln2 with ln2 split into a short high part (exact product) and a low
//  correction (Cody & Waite 1980); exp(r) on |r| <= ln2/2 by the degree-7 Taylor series in Horner form
//  (truncation < 6e-9 relative); scale by 2^n through the exponent field.  Only fmaf, mul, add and
//  integer ops are used, each correctly rounded, so every platform returns the same bits.
//  x is clamped to [-86, 88] so 2^n stays a normal float (exp(-86) ~ 4e-38, exp(88) ~ 1.7e38).
LK_HD float lk_expf(float x) {
    x = x < -86.0f ? -86.0f : (x > 88.0f ? 88.0f : x);
    const float LOG2E = 1.44269504088896341f;
    const float LN2_HI = 0.693145751953125f;          // 0x3F317200: 16 significant bits, n*LN2_HI exact
    const float LN2_LO = 1.42860676533018740e-06f;    // ln2 - LN2_HI
    const float n = rintf(x * LOG2E);
    float r = fmaf(-n, LN2_HI, x);
    r = fmaf(-n, LN2_LO, r);
    float p = 1.0f / 5040.0f;
    p = fmaf(p, r, 1.0f / 720.0f);
    p = fmaf(p, r, 1.0f / 120.0f);
    p = fmaf(p, r, 1.0f / 24.0f);
    p = fmaf(p, r, 1.0f / 6.0f);
    p = fmaf(p, r, 0.5f);
    p = fmaf(p, r, 1.0f);
    p = fmaf(p, r, 1.0f);
    const int ni = (int)n;
    return p * bits_f32((uint32_t)(ni + 127) << 23);
}

// sigmoid as the router uses it: 1 / (1 + exp(-v)) (fused_layer.cu:321), with lk_expf.
LK_HD float lk_sigmoid(float v) { return 1.0f / (1.0f + lk_expf(-v)); }
// silu(g) * u as SwiGLU uses it: g / (1 + exp(-g)) * u (fused_layer.cu:337), with lk_expf.
LK_HD float lk_swiglu(float g, float u) { return g / (1.0f + lk_expf(-g)) * u; }

// ---- q8 per 32 (fused_layer.cu:40-47): d = amax/127, q = round-half-even(x / d) via x * (1/d)
//  Returns d; q[0..32) receive the int8 values.  Round-half-even is rintf under the default rounding
//  mode on the host and __float2int_rn on the device; both are exact functions of (x*id).
LK_HD float quant_q8_group(const float* x, int8_t* q) {
    float amax = 0.0f;
    for (int j = 0; j < 32; ++j) { const float a = fabsf(x[j]); amax = amax > a ? amax : a; }
    const float d = amax / 127.0f, id = d > 0.0f ? 1.0f / d : 0.0f;
    for (int j = 0; j < 32; ++j) q[j] = (int8_t)(int)rintf(x[j] * id);
    return d;
}

// ---- IQ2_XXS group helpers.  A 66-byte block = fp16 d, then 8 groups of 8 bytes; group s of a block =
//  bytes [2+8s, 10+8s): aux0 (4 grid indices, one per 8-weight sub-group) and aux1 (4 x 7-bit sign
//  indices in bits 0..27, 4-bit scale in bits 28..31).  Weight value = d * (0.5 + scale) * 0.25 *
//  grid[idx][j] * sign, sign bits = ksigns(sign index) (gguf-py IQ2_XXS.dequantize_blocks; the
//  reference's iq2_unpack4, fused_layer.cu:30-33, and its scale, :191).
LK_HD uint32_t iq2_ksigns(uint32_t i7) {           // 7 stored sign bits + even-parity bit 7
    uint32_t p = i7 ^ (i7 >> 4); p ^= p >> 2; p ^= p >> 1;
    return i7 | ((p & 1u) << 7);
}

// ---- seeded synthetic IQ2_XXS weights (counter-based; the same bytes on CPU and GPU)
//  key chain: seed -> layer -> matrix (0 gate, 1 up, 2 down) -> expert (256 = shared expert);
//  block b of the matrix (b = row * (K/256) + column block): 8 x splitmix64 draws give the 8 groups'
//  64 bits verbatim (every bit pattern is a valid grid index / sign index / scale: uniform fields),
//  3 more draws give 12 x 16-bit uniforms whose Irwin-Hall sum approximates N(0,1); d = fp16(|N|*1e-3).
LK_HD uint64_t splitmix64(uint64_t x) {
    x += 0x9E3779B97F4A7C15ull;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
    return x ^ (x >> 31);
}
LK_HD uint64_t iq2_gen_key(uint64_t seed, uint32_t layer, uint32_t matrix, uint32_t expert) {
    uint64_t h = splitmix64(seed);
    h = splitmix64(h ^ (uint64_t)layer);
    h = splitmix64(h ^ ((uint64_t)matrix << 32));
    return splitmix64(h ^ ((uint64_t)expert << 16));
}
// fp16(|N(0,1)| * scale) from the draws at block*16 + 8..10
LK_HD uint16_t gen_abs_normal_half(uint64_t key, uint64_t block, float scale) {
    int32_t s = 0;
    for (int w = 0; w < 3; ++w) {
        const uint64_t r = splitmix64(key ^ (block * 16ull + 8ull + (uint64_t)w));
        for (int j = 0; j < 4; ++j) s += (int32_t)((r >> (16 * j)) & 0xFFFFull);
    }
    const int32_t c = 2 * s - 12 * 65535;            // 2 * (sum - 12 * 65535/2): exact integer
    const float n = (float)c * (1.0f / 131072.0f);   // / 2^17: unit-variance Irwin-Hall(12), exact
    const float a = fabsf(n) * scale;
    return float_to_half_rne(a);
}
LK_HD uint16_t iq2_gen_d(uint64_t key, uint64_t block) { return gen_abs_normal_half(key, block, 1.0e-3f); }
LK_HD uint64_t iq2_gen_group(uint64_t key, uint64_t block, int g) {
    return splitmix64(key ^ (block * 16ull + (uint64_t)g));
}
// write block `block` (66 bytes) of the matrix identified by key
LK_HD void iq2_gen_block(uint64_t key, uint64_t block, uint8_t* out) {
    const uint16_t d = iq2_gen_d(key, block);
    out[0] = (uint8_t)(d & 0xFF); out[1] = (uint8_t)(d >> 8);
    for (int g = 0; g < 8; ++g) {
        const uint64_t v = iq2_gen_group(key, block, g);
        for (int j = 0; j < 8; ++j) out[2 + 8 * g + j] = (uint8_t)(v >> (8 * j));
    }
}

// seeded synthetic K-quant blocks (Q2_K / Q3_K downs, Q5_K / Q6_K shared expert): every byte except the
// fp16 scales is uniform (splitmix64 draws 0..26 of the block's counter range, 8 bytes each), d =
// fp16(|N(0,1)|*c) from the draws at block*2 + 2^40, dmin (Q2_K, Q5_K) from block*2 + 1 + 2^40; c = 1e-3
// (Q2_K, Q3_K) or 4e-5 (Q5_K, Q6_K, whose 5- and 6-bit values and 6- and 8-bit scales are ~30-100x wider),
// so every format's weights have the IQ2_XXS experts' magnitude.  Keys as for IQ2_XXS, so a layer's matrix
// in any format comes from the same (seed, layer, matrix, expert) chain.
LK_HD void kq_gen_block(int fmt, uint64_t key, uint64_t block, uint8_t* out) {
    const int nb = fmt_block_bytes(fmt);
    for (int g = 0; 8 * g < nb; ++g) {
        const uint64_t v = splitmix64(key ^ (block * 32ull + (uint64_t)g));
        for (int j = 0; j < 8 && 8 * g + j < nb; ++j) out[8 * g + j] = (uint8_t)(v >> (8 * j));
    }
    const int doff = fmt == FMT_Q2K ? Q2K_D : fmt == FMT_Q3K ? Q3K_D : fmt == FMT_Q6K ? Q6K_D : 0;
    const float c = (fmt == FMT_Q5K || fmt == FMT_Q6K) ? 4.0e-5f : 1.0e-3f;
    const uint16_t d = gen_abs_normal_half(key, block * 2ull + (1ull << 40), c);
    out[doff] = (uint8_t)(d & 0xFF); out[doff + 1] = (uint8_t)(d >> 8);
    if (fmt == FMT_Q2K || fmt == FMT_Q5K) {
        const int moff = fmt == FMT_Q2K ? Q2K_DMIN : 2;
        const uint16_t m = gen_abs_normal_half(key, block * 2ull + 1ull + (1ull << 40), c);
        out[moff] = (uint8_t)(m & 0xFF); out[moff + 1] = (uint8_t)(m >> 8);
    }
}

}  // namespace lk
