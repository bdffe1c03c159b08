// oracle.cpp -- CPU restatement of loki's MoE hot path.  TEST INFRASTRUCTURE ONLY: tests/, the smoke
// check and bench.py's CPU-baseline leg load it as the checker; the product never links or calls it.
//
// Parity anchors (reference = grimnier/loki, paths inside that project):
//   IQ2_XXS decode ........ src/fused_layer.cu:30-33 (iq2_unpack4), :185-191 (block walk, scale d*(0.5+s)*0.25);
//                           cross-checked against gguf-py 0.19.0 gguf.quants.IQ2_XXS.dequantize_blocks
//   q8 activations ........ src/fused_layer.cu:40-47 (quant_x: d = amax/127, q = rint(x/d) half-even)
//   router ................ src/fused_layer.cu:314-332 (sigmoid(W.x), top-8 of p+bias, ties -> lower id,
//                           w = p/max(sum p, 2^-14) * 2.5); src/server_core_fused.cpp:646-651 (ggml twin)
//   grouped top-k ......... not in the reference (the BASELINE's DeepSeek-V3 mode): n_group groups of
//                           consecutive experts, group score = sum of its top-2 (p+bias), keep topk_group
//                           groups, top-k inside them
//   keep-KE + renorm ...... src/server_core_fused.cpp:793-813 (sort by w desc, keep KE, scale to sum 2.5)
//   SwiGLU + q8 ........... src/fused_layer.cu:334-341 (h = g/(1+exp(-g))*u, re-quantised per 32)
//   expert products ....... src/fused_layer.cu:178-202 (IQ2 gate/up/down: sum_g fa_g * dx_g * isum_g)
//   K-quant downs ......... src/fused_layer.cu:203-227 (Q2_K: per 16 weights fa*dx*isum - dmin*m*s16),
//                           :228-254 (Q3_K: fa = d*(scale-32), q = low2 - 4 where the high bit is clear);
//                           block decode cross-checked against gguf-py 0.19.0 Q2_K / Q3_K dequantize
//   shared expert ......... src/fused_layer.cu:521-524 with tc_matvec's Q5_K (:102-130, per 32 weights
//                           fa*dx*isum - dmin*m*sx) and Q6_K (:131-158, per 16 weights) arithmetic; block
//                           decode cross-checked against gguf-py 0.19.0 Q5_K / Q6_K dequantize
//   combine ............... src/fused_layer.cu:366-373 and 354-360 (routed = sum_k w_k y_k; h = routed +
//                           shared + ffn_inp; moe = routed)
//
// Pinned against the reference's own kernels: oracle/_ref/libref_moe.so (src/fused_layer.cu built from its
// sources by `make ref`) runs the router, the Q5_K/Q6_K shared expert and fl_moe on the GPU, and
// tests/test_gpu_ref_pin.py holds this file's router (ids equal, weights within 2e-6) and layer outputs
// (within 1e-4 relative L2; measured ~2.3e-7) to them.
//   permute ............... src/server_core_fused.cpp:937 (byexp: per expert, (row, k) pairs in row-major
//                           order) -- the per-expert token lists, stable by (token, k)
//
// Arithmetic: the router logits follow the GPU kernel's fixed reduction order exactly (see
// orc_router_logits), and exp is lk_expf from moe_format.h on both sides, so router probabilities,
// selected ids and weights are bit-identical to the kernels.  Expert products are evaluated in double
// from the same quantised operands (integer group sums are exact), i.e. the ideal value of the q8
// scheme; the kernels' fp32 accumulation differs from it by reassociation only.
#include <cstdint>
#include <cstring>
#include <cmath>
#include <vector>
#include <algorithm>
#include "../loki_b200/csrc/moe_format.h"

using namespace lk;

static const uint64_t IQ2_GRID[256] = {
#include "../loki_b200/csrc/iq2_grid.inc"
};

extern "C" {

// ------------------------------------------------------------------ formats
// out[rows*K] = dequantised IQ2_XXS weights (gguf-py dequantize_blocks semantics)
static void iq2_deq_block(const uint8_t* blk, float* out) {
    uint16_t dh; memcpy(&dh, blk, 2);
    const float d = half_to_float(dh);
    for (int g = 0; g < 8; ++g) {
        uint32_t aux0, aux1; memcpy(&aux0, blk + 2 + 8 * g, 4); memcpy(&aux1, blk + 6 + 8 * g, 4);
        const float db = d * (0.5f + (float)(aux1 >> 28)) * 0.25f;
        for (int l = 0; l < 4; ++l) {
            const uint64_t gv = IQ2_GRID[(aux0 >> (8 * l)) & 0xFF];
            const uint32_t s = iq2_ksigns((aux1 >> (7 * l)) & 127u);
            for (int j = 0; j < 8; ++j) {
                const float m = (float)((gv >> (8 * j)) & 0xFF);
                out[g * 32 + l * 8 + j] = db * m * ((s >> j) & 1 ? -1.0f : 1.0f);
            }
        }
    }
}

void orc_iq2_dequant(const uint8_t* blocks, int64_t nblk, float* out) {
    #pragma omp parallel for schedule(static)
    for (int64_t b = 0; b < nblk; ++b) iq2_deq_block(blocks + b * BLK_IQ2, out + b * 256);
}

// seeded generator (moe_format.h): rows x K matrix of (layer, matrix, expert)
void orc_gen_iq2(uint64_t seed, int layer, int matrix, int expert, int rows, int K, uint8_t* out) {
    const uint64_t key = iq2_gen_key(seed, (uint32_t)layer, (uint32_t)matrix, (uint32_t)expert);
    const int64_t nblk = (int64_t)rows * (K / QK);
    #pragma omp parallel for schedule(static)
    for (int64_t b = 0; b < nblk; ++b) iq2_gen_block(key, (uint64_t)b, out + b * BLK_IQ2);
}

void orc_gen_d_only(uint64_t seed, int layer, int matrix, int expert, int64_t nblk, uint16_t* out) {
    const uint64_t key = iq2_gen_key(seed, (uint32_t)layer, (uint32_t)matrix, (uint32_t)expert);
    for (int64_t b = 0; b < nblk; ++b) out[b] = iq2_gen_d(key, (uint64_t)b);
}

// out[nblk*256] = dequantised Q2_K (fmt 5), Q3_K (6), Q5_K (3) or Q6_K (1) blocks (gguf-py
// dequantize_blocks semantics: Q2_K d*(sc&15)*q - dmin*(sc>>4); Q3_K d*(scale-32)*q3; Q5_K
// (d*scale)*q - dmin*min; Q6_K (d*scale)*(q-32); each product in fp32 as written)
static void kq_deq_block(int fmt, const uint8_t* blk, float* out) {
    if (fmt == FMT_Q5K) {
        uint16_t dh, mh; memcpy(&dh, blk, 2); memcpy(&mh, blk + 2, 2);
        const float d = half_to_float(dh), dmin = half_to_float(mh);
        for (int i = 0; i < QK; ++i) {
            const int j = i >> 6, u = (i >> 5) & 1, l = i & 31;
            const int q = ((blk[Q5K_QS + 32 * j + l] >> (4 * u)) & 15) | (((blk[Q5K_QH + l] >> (2 * j + u)) & 1) << 4);
            int sc, mn; q5k_scale_min(blk + Q5K_SC, 2 * j + u, sc, mn);
            out[i] = (d * (float)sc) * (float)q - dmin * (float)mn;
        }
        return;
    }
    if (fmt == FMT_Q6K) {
        uint16_t dh; memcpy(&dh, blk + Q6K_D, 2);
        const float d = half_to_float(dh);
        for (int i = 0; i < QK; ++i) {
            const int n = i >> 7, c = (i >> 5) & 3, l = i & 31;
            const int q = ((blk[64 * n + 32 * (c & 1) + l] >> (4 * (c >> 1))) & 15) | (((blk[Q6K_QH + 32 * n + l] >> (2 * c)) & 3) << 4);
            out[i] = (d * (float)(int8_t)blk[Q6K_SC + i / 16]) * (float)(q - 32);
        }
        return;
    }
    for (int i = 0; i < QK; ++i) {
        const int n = i >> 7, j = (i >> 5) & 3, s = (i >> 4) & 1, l = i & 15;
        const int is = 8 * n + 2 * j + s;
        float v;
        if (fmt == FMT_Q2K) {
            uint16_t dh, mh; memcpy(&dh, blk + Q2K_D, 2); memcpy(&mh, blk + Q2K_DMIN, 2);
            const int q = (blk[Q2K_QS + 32 * n + 16 * s + l] >> (2 * j)) & 3;
            const float dl = half_to_float(dh) * (float)(blk[is] & 15), ml = half_to_float(mh) * (float)(blk[is] >> 4);
            v = dl * (float)q - ml;
        } else {
            uint16_t dh; memcpy(&dh, blk + Q3K_D, 2);
            const int lo = (blk[Q3K_QS + 32 * n + 16 * s + l] >> (2 * j)) & 3;
            const int hb = (blk[16 * s + l] >> (4 * n + j)) & 1;
            const float dl = half_to_float(dh) * (float)q3k_scale(blk + Q3K_SC, is);
            v = dl * (float)(lo - (hb ? 0 : 4));
        }
        out[i] = v;
    }
}

void orc_kq_dequant(int fmt, const uint8_t* blocks, int64_t nblk, float* out) {
    const int nb = fmt_block_bytes(fmt);
    #pragma omp parallel for schedule(static)
    for (int64_t b = 0; b < nblk; ++b) kq_deq_block(fmt, blocks + b * nb, out + b * QK);
}

// seeded K-quant matrix (moe_format.h kq_gen_block): rows x K in format fmt of (layer, matrix, expert)
void orc_gen_kq(int fmt, uint64_t seed, int layer, int matrix, int expert, int rows, int K, uint8_t* out) {
    const uint64_t key = iq2_gen_key(seed, (uint32_t)layer, (uint32_t)matrix, (uint32_t)expert);
    const int64_t nblk = (int64_t)rows * (K / QK);
    const int nb = fmt_block_bytes(fmt);
    #pragma omp parallel for schedule(static)
    for (int64_t b = 0; b < nblk; ++b) kq_gen_block(fmt, key, (uint64_t)b, out + b * nb);
}

float orc_expf(float x) { return lk_expf(x); }
uint16_t orc_f2h(float x) { return float_to_half_rne(x); }
float orc_h2f(uint16_t h) { return half_to_float(h); }

// q8 per 32 of n values (n % 32 == 0): q[n], d[n/32]
void orc_quant_q8(const float* x, int64_t n, int8_t* q, float* d) {
    for (int64_t g = 0; g < n / 32; ++g) d[g] = quant_q8_group(x + g * 32, q + g * 32);
}

// ------------------------------------------------------------------ router
// logits[t][e] = W[e] . x[t] in the GPU router kernel's order: 256 partial sums per (t, e); partial p
// (p = 32*warp + lane, 8 warps) runs over float4 chunks c = p, p+256, ... (7 chunks for 7168) and within a
// chunk over its 4 components, each step acc = fmaf(w, x, acc); each warp's 32 partials are combined by the
// xor butterfly (offsets 16, 8, 4, 2, 1: a_l <- a_l + a_(l^o)); the 8 warp sums as
// ((s0 + s1) + (s2 + s3)) + ((s4 + s5) + (s6 + s7)).
void orc_router_logits(const float* x, int T, const float* W, int n_experts, int K, float* logits) {
    const int NCH = K / 4;
    #pragma omp parallel for collapse(2) schedule(static)
    for (int t = 0; t < T; ++t)
        for (int e = 0; e < n_experts; ++e) {
            const float* xr = x + (size_t)t * K; const float* wr = W + (size_t)e * K;
            float ws[8];
            for (int w = 0; w < 8; ++w) {
                float a[32];
                for (int l = 0; l < 32; ++l) {
                    float acc = 0.0f;
                    for (int c = 32 * w + l; c < NCH; c += 256)
                        for (int j = 0; j < 4; ++j) acc = fmaf(wr[4 * c + j], xr[4 * c + j], acc);
                    a[l] = acc;
                }
                for (int o = 16; o > 0; o >>= 1) {
                    float b[32];
                    for (int l = 0; l < 32; ++l) b[l] = a[l] + a[l ^ o];
                    memcpy(a, b, sizeof(a));
                }
                ws[w] = a[0];
            }
            logits[(size_t)t * n_experts + e] = ((ws[0] + ws[1]) + (ws[2] + ws[3])) + ((ws[4] + ws[5]) + (ws[6] + ws[7]));
        }
}

struct OrcRouteCfg {
    int n_experts;    // 256
    int topk;         // experts selected by score (8)
    int keep;         // experts kept per token after the weight sort (KE <= topk)
    int renorm;       // 1: kept weights rescaled to sum to `scale` (engine default)
    int n_group;      // 1 = plain top-k (the reference); 8 = DeepSeek-V3 grouped
    int topk_group;   // groups kept in grouped mode (4)
    float scale;      // routed scaling factor (2.5)
};

// one token: probs[n_experts] -> sel[keep], w[keep]
static void route_one(const float* p, const float* bias, const OrcRouteCfg& c, int* sel, float* w) {
    const int NE = c.n_experts;
    std::vector<float> sc(NE);
    for (int e = 0; e < NE; ++e) sc[e] = p[e] + bias[e];
    std::vector<char> allowed(NE, 1);
    if (c.n_group > 1) {
        const int gs = NE / c.n_group;
        std::vector<float> gscore(c.n_group);
        for (int g = 0; g < c.n_group; ++g) {   // top-2 of the group (ties -> lower id), summed larger-first
            int i1 = -1, i2 = -1;
            for (int e = g * gs; e < (g + 1) * gs; ++e) {
                if (i1 < 0 || sc[e] > sc[i1]) { i2 = i1; i1 = e; }
                else if (i2 < 0 || sc[e] > sc[i2]) i2 = e;
            }
            gscore[g] = sc[i1] + sc[i2];
        }
        std::vector<char> gkeep(c.n_group, 0);
        for (int r = 0; r < c.topk_group; ++r) {
            int bg = -1;
            for (int g = 0; g < c.n_group; ++g) if (!gkeep[g] && (bg < 0 || gscore[g] > gscore[bg])) bg = g;
            gkeep[bg] = 1;
        }
        for (int e = 0; e < NE; ++e) allowed[e] = gkeep[e / gs];
    }
    int top[MAX_TOPK]; std::vector<char> taken(NE, 0);
    for (int k = 0; k < c.topk; ++k) {                    // argmax rounds, ties -> lower id
        int bi = -1;
        for (int e = 0; e < NE; ++e) if (allowed[e] && !taken[e] && (bi < 0 || sc[e] > sc[bi])) bi = e;
        top[k] = bi; taken[bi] = 1;
    }
    float sum = 0.0f;
    for (int k = 0; k < c.topk; ++k) sum += p[top[k]];
    sum = fmaxf(sum, 6.103515625e-5f);
    float wt[MAX_TOPK];
    for (int k = 0; k < c.topk; ++k) wt[k] = p[top[k]] / sum * c.scale;
    if (c.keep >= c.topk) { for (int k = 0; k < c.topk; ++k) { sel[k] = top[k]; w[k] = wt[k]; } return; }
    int ord[MAX_TOPK]; for (int k = 0; k < c.topk; ++k) ord[k] = k;
    std::stable_sort(ord, ord + c.topk, [&](int a, int b) { return wt[a] > wt[b]; });   // ties keep position order
    float kw[MAX_TOPK]; float sw = 0.0f;
    for (int k = 0; k < c.keep; ++k) { sel[k] = top[ord[k]]; kw[k] = wt[ord[k]]; sw += kw[k]; }
    if (c.renorm && sw > 1e-6f) { const float f = c.scale / sw; for (int k = 0; k < c.keep; ++k) kw[k] *= f; }
    for (int k = 0; k < c.keep; ++k) w[k] = kw[k];
}

// probs may be null; logits_in: optional precomputed logits (replaces W.x; the "uniform-random logits" mode)
void orc_router(const float* x, int T, const float* W, const float* logits_in, const float* bias,
                const OrcRouteCfg* cfg, float* probs_out, int* sel, float* w) {
    const int NE = cfg->n_experts;
    std::vector<float> logit((size_t)T * NE);
    if (logits_in) memcpy(logit.data(), logits_in, logit.size() * 4);
    else orc_router_logits(x, T, W, NE, HIDDEN, logit.data());
    std::vector<float> p(logit.size());
    for (size_t i = 0; i < p.size(); ++i) p[i] = lk_sigmoid(logit[i]);
    if (probs_out) memcpy(probs_out, p.data(), p.size() * 4);
    #pragma omp parallel for schedule(static)
    for (int t = 0; t < T; ++t) route_one(&p[(size_t)t * NE], bias, *cfg, sel + (size_t)t * cfg->keep, w + (size_t)t * cfg->keep);
}

// ------------------------------------------------------------------ permute (dispatch order)
// counts[NE], offsets[NE+1], perm[T*KE] = flat (t*KE + k) indices grouped by expert, stable by (t, k)
void orc_permute(const int* sel, int T, int KE, int NE, int* counts, int* offsets, int* perm) {
    for (int e = 0; e < NE; ++e) counts[e] = 0;
    for (int i = 0; i < T * KE; ++i) counts[sel[i]]++;
    offsets[0] = 0;
    for (int e = 0; e < NE; ++e) offsets[e + 1] = offsets[e] + counts[e];
    std::vector<int> fill(offsets, offsets + NE);
    for (int i = 0; i < T * KE; ++i) perm[fill[sel[i]]++] = i;
}

// ------------------------------------------------------------------ expert products
// integer dot of IQ2 group g of a row with 32 q8 activations
static inline int32_t iq2_group_isum(const uint8_t* grp, const int8_t* xq) {
    uint32_t aux0, aux1; memcpy(&aux0, grp, 4); memcpy(&aux1, grp + 4, 4);
    int32_t s = 0;
    for (int l = 0; l < 4; ++l) {
        const uint64_t gv = IQ2_GRID[(aux0 >> (8 * l)) & 0xFF];
        const uint32_t sg = iq2_ksigns((aux1 >> (7 * l)) & 127u);
        for (int j = 0; j < 8; ++j) {
            const int32_t m = (int32_t)((gv >> (8 * j)) & 0xFF);
            s += ((sg >> j) & 1 ? -m : m) * (int32_t)xq[8 * l + j];
        }
    }
    return s;
}

// y = W . dequant(xq, xd) for `ntok` activation rows (each K int8 + K/32 scales), W = rows x K IQ2_XXS
static void iq2_matvec_multi(const uint8_t* W, int rows, int K, const int8_t* const* xq, const float* const* xd,
                             int ntok, float* const* y) {
    const int NB = K / QK;
    #pragma omp parallel for schedule(static)
    for (int r = 0; r < rows; ++r) {
        const uint8_t* row = W + (size_t)r * NB * BLK_IQ2;
        std::vector<double> acc(ntok, 0.0);
        for (int b = 0; b < NB; ++b) {
            const uint8_t* blk = row + (size_t)b * BLK_IQ2;
            uint16_t dh; memcpy(&dh, blk, 2); const float d = half_to_float(dh);
            for (int g = 0; g < 8; ++g) {
                uint32_t aux1; memcpy(&aux1, blk + 6 + 8 * g, 4);
                const float fa = d * (0.5f + (float)(aux1 >> 28)) * 0.25f;
                const int col = b * 8 + g;
                for (int t = 0; t < ntok; ++t) {
                    const int32_t is = iq2_group_isum(blk + 2 + 8 * g, xq[t] + col * 32);
                    acc[t] += (double)fa * (double)xd[t][col] * (double)is;
                }
            }
        }
        for (int t = 0; t < ntok; ++t) y[t][r] = (float)acc[t];
    }
}

// y = W . h for fp32 activations h (no q8): the tensor-core path's down projection, which consumes the
// SwiGLU output at 16-bit precision instead of re-quantising it
static void iq2_matvec_float_multi(const uint8_t* W, int rows, int K, const float* const* h, int ntok, float* const* y) {
    const int NB = K / QK;
    #pragma omp parallel for schedule(static)
    for (int r = 0; r < rows; ++r) {
        const uint8_t* row = W + (size_t)r * NB * BLK_IQ2;
        std::vector<double> acc(ntok, 0.0);
        for (int b = 0; b < NB; ++b) {
            const uint8_t* blk = row + (size_t)b * BLK_IQ2;
            uint16_t dh; memcpy(&dh, blk, 2); const float d = half_to_float(dh);
            for (int g = 0; g < 8; ++g) {
                uint32_t aux0, aux1; memcpy(&aux0, blk + 2 + 8 * g, 4); memcpy(&aux1, blk + 6 + 8 * g, 4);
                const double fa = (double)(d * (0.5f + (float)(aux1 >> 28)) * 0.25f);
                for (int l = 0; l < 4; ++l) {
                    const uint64_t gv = IQ2_GRID[(aux0 >> (8 * l)) & 0xFF];
                    const uint32_t sg = iq2_ksigns((aux1 >> (7 * l)) & 127u);
                    for (int j = 0; j < 8; ++j) {
                        const int32_t m = (int32_t)((gv >> (8 * j)) & 0xFF);
                        const int32_t wv = (sg >> j) & 1 ? -m : m;
                        const int k = b * 256 + g * 32 + l * 8 + j;
                        for (int t = 0; t < ntok; ++t) acc[t] += fa * (double)wv * (double)h[t][k];
                    }
                }
            }
        }
        for (int t = 0; t < ntok; ++t) y[t][r] = (float)acc[t];
    }
}

// y = W . dequant(xq, xd) for a K-quant matrix (Q2_K / Q3_K) and `ntok` q8 activation rows, in the
// reference's per-16 arithmetic (src/fused_layer.cu:203-254): per 16-weight sub-block an exact integer
// sum isum = sum q_w * q_x; Q2_K adds fa*dx*isum - mla*dx*sum(q_x) with fa = d*(sc&15), mla = dmin*(sc>>4)
// (the reference's s16 term); Q3_K adds fa*dx*isum with fa = d*(scale-32) and q_w = low2 - 4 where the
// high bit is clear.  Evaluated in double: the ideal value of the q8 scheme.
//
// Q5_K (the shared expert's gate/up, src/fused_layer.cu:102-130): per 32-weight sub-block isum = sum q_w * q_x
// (q_w in 0..31), acc += dx * (d*scale*isum - dmin*min*sum q_x).  Q6_K (the shared down, :131-158): per
// 16-weight sub-block isum = sum (q_w - 32) * q_x, acc += d*scales[i/16]*dx*isum.
static void q56_matvec_multi(int fmt, const uint8_t* W, int rows, int K, const int8_t* const* xq, const float* const* xd,
                             int ntok, float* const* y) {
    const int NB = K / QK, nb = fmt_block_bytes(fmt);
    #pragma omp parallel for schedule(static)
    for (int r = 0; r < rows; ++r) {
        const uint8_t* row = W + (size_t)r * NB * nb;
        std::vector<double> acc(ntok, 0.0);
        for (int b = 0; b < NB; ++b) {
            const uint8_t* blk = row + (size_t)b * nb;
            if (fmt == FMT_Q5K) {
                uint16_t dh, mh; memcpy(&dh, blk, 2); memcpy(&mh, blk + 2, 2);
                const double d = half_to_float(dh), dmin = half_to_float(mh);
                for (int sb = 0; sb < 8; ++sb) {
                    const int j = sb >> 1, u = sb & 1, k0 = b * QK + 32 * sb;
                    int sc, mn; q5k_scale_min(blk + Q5K_SC, sb, sc, mn);
                    int32_t qw[32];
                    for (int l = 0; l < 32; ++l)
                        qw[l] = ((blk[Q5K_QS + 32 * j + l] >> (4 * u)) & 15) | (((blk[Q5K_QH + l] >> (2 * j + u)) & 1) << 4);
                    for (int t = 0; t < ntok; ++t) {
                        int32_t isum = 0, xs = 0;
                        for (int l = 0; l < 32; ++l) { isum += qw[l] * (int32_t)xq[t][k0 + l]; xs += xq[t][k0 + l]; }
                        acc[t] += (double)xd[t][k0 / 32] * (d * sc * (double)isum - dmin * mn * (double)xs);
                    }
                }
            } else {
                uint16_t dh; memcpy(&dh, blk + Q6K_D, 2);
                const double d = half_to_float(dh);
                for (int s16 = 0; s16 < 16; ++s16) {
                    const int k0 = b * QK + 16 * s16;
                    int32_t qw[16];
                    for (int l = 0; l < 16; ++l) {
                        const int i = 16 * s16 + l, n = i >> 7, c = (i >> 5) & 3, ll = i & 31;
                        qw[l] = (((blk[64 * n + 32 * (c & 1) + ll] >> (4 * (c >> 1))) & 15) |
                                 (((blk[Q6K_QH + 32 * n + ll] >> (2 * c)) & 3) << 4)) - 32;
                    }
                    const double fa = d * (double)(int8_t)blk[Q6K_SC + s16];
                    for (int t = 0; t < ntok; ++t) {
                        int32_t isum = 0;
                        for (int l = 0; l < 16; ++l) isum += qw[l] * (int32_t)xq[t][k0 + l];
                        acc[t] += fa * (double)xd[t][k0 / 32] * (double)isum;
                    }
                }
            }
        }
        for (int t = 0; t < ntok; ++t) y[t][r] = (float)acc[t];
    }
}

static void kq_matvec_multi(int fmt, const uint8_t* W, int rows, int K, const int8_t* const* xq, const float* const* xd,
                            int ntok, float* const* y) {
    if (fmt == FMT_Q5K || fmt == FMT_Q6K) { q56_matvec_multi(fmt, W, rows, K, xq, xd, ntok, y); return; }
    const int NB = K / QK, nb = fmt_block_bytes(fmt);
    const int qs = fmt == FMT_Q2K ? Q2K_QS : Q3K_QS;
    #pragma omp parallel for schedule(static)
    for (int r = 0; r < rows; ++r) {
        const uint8_t* row = W + (size_t)r * NB * nb;
        std::vector<double> acc(ntok, 0.0);
        for (int b = 0; b < NB; ++b) {
            const uint8_t* blk = row + (size_t)b * nb;
            uint16_t dh, mh = 0;
            memcpy(&dh, blk + (fmt == FMT_Q2K ? Q2K_D : Q3K_D), 2);
            if (fmt == FMT_Q2K) memcpy(&mh, blk + Q2K_DMIN, 2);
            const float d = half_to_float(dh), dmin = half_to_float(mh);
            for (int is = 0; is < 16; ++is) {                     // sub-block 8n + 2j + s
                const int n = is >> 3, j = (is >> 1) & 3, s = is & 1;
                const int k0 = b * QK + 128 * n + 32 * j + 16 * s;
                int32_t qw[16];
                for (int l = 0; l < 16; ++l) {
                    const int lo = (blk[qs + 32 * n + 16 * s + l] >> (2 * j)) & 3;
                    qw[l] = fmt == FMT_Q2K ? lo : lo - (((blk[16 * s + l] >> (4 * n + j)) & 1) ? 0 : 4);
                }
                const double fa = fmt == FMT_Q2K ? (double)(d * (float)(blk[is] & 15)) : (double)(d * (float)q3k_scale(blk + Q3K_SC, is));
                const double mla = fmt == FMT_Q2K ? (double)(dmin * (float)(blk[is] >> 4)) : 0.0;
                for (int t = 0; t < ntok; ++t) {
                    int32_t isum = 0, xs = 0;
                    for (int l = 0; l < 16; ++l) { isum += qw[l] * (int32_t)xq[t][k0 + l]; xs += xq[t][k0 + l]; }
                    const double dx = (double)xd[t][k0 / 32];
                    acc[t] += fa * dx * (double)isum - mla * dx * (double)xs;
                }
            }
        }
        for (int t = 0; t < ntok; ++t) y[t][r] = (float)acc[t];
    }
}

// y = W . h for a K-quant matrix and `ntok` unquantised activation rows: every row dequantised as gguf-py
// does (orc_kq_dequant), the dot products in double.  The reference for the kernels that keep the SwiGLU
// output at 16-bit precision (the mma.sync K-quant down).
static void kq_matvec_float_multi(int fmt, const uint8_t* W, int rows, int K, const float* const* h, int ntok, float* const* y) {
    const int NB = K / QK, nb = fmt_block_bytes(fmt);
    #pragma omp parallel for schedule(static)
    for (int r = 0; r < rows; ++r) {
        std::vector<float> wr((size_t)K);
        for (int b = 0; b < NB; ++b) orc_kq_dequant(fmt, W + ((size_t)r * NB + b) * nb, 1, wr.data() + (size_t)b * QK);
        for (int t = 0; t < ntok; ++t) {
            double acc = 0.0;
            for (int k = 0; k < K; ++k) acc += (double)wr[k] * (double)h[t][k];
            y[t][r] = (float)acc;
        }
    }
}

// one activation row through a K-quant matrix (tests)
void orc_kq_matvec(int fmt, const uint8_t* W, int rows, int K, const int8_t* xq, const float* xd, float* y) {
    kq_matvec_multi(fmt, W, rows, K, &xq, &xd, 1, &y);
}

void orc_iq2_matvec(const uint8_t* W, int rows, int K, const int8_t* xq, const float* xd, float* y) {
    iq2_matvec_multi(W, rows, K, &xq, &xd, 1, &y);
}

// ------------------------------------------------------------------ the MoE layer
// Weights in the engine's arena layout: expert m's gate at gate + m*gate_stride (bytes), likewise up/down;
// ids are expert (slot) indices into those arenas.  Shared expert (IQ2_XXS) optional (null = none).
// Outputs: h[T][E] = routed + shared + resid, moe[T][E] = routed; optional y_slot[T][KE][E] (w-weighted
// per-slot outputs, the reference's out_all), hq/hd: SwiGLU q8 per (t, k) slot [T*KE][2048] / [T*KE][64].
struct OrcLayerW {
    const uint8_t* gate; const uint8_t* up; const uint8_t* down; int64_t gate_stride, up_stride, down_stride;
    const uint8_t* sh_gate; const uint8_t* sh_up; const uint8_t* sh_down;
};

// hq8 = 1: the SwiGLU output is re-quantised to q8 per 32 before the down projection (the reference's
// swiglu_q8, src/fused_layer.cu:334-341: the decode and narrow paths); hq8 = 0: it enters the down
// projection unquantised (the tensor-core prefill path).
// down_fmt: format of every routed down matrix (FMT_IQ2, FMT_Q2K or FMT_Q3K; with hq8 = 1 the K-quants use
// the reference's per-16 q8 arithmetic, with hq8 = 0 the unquantised h against the dequantised rows).  The shared expert's gate/up are in sh_gu_fmt (FMT_IQ2, or the
// real model's FMT_Q5K) and its down in sh_down_fmt (down_fmt, or FMT_Q6K); its SwiGLU output is always
// re-quantised to q8 when either is a K-quant (the reference's shared path, fused_layer.cu:521-524).
int orc_moe_layer_fmt2(const float* x, const float* resid, int T, const OrcLayerW* Wl, const int* ids, const float* w,
                       int KE, float* h, float* moe, float* y_slot, float* shared_out, int hq8, int down_fmt,
                       int sh_gu_fmt, int sh_down_fmt) {
    if (down_fmt != FMT_IQ2 && down_fmt != FMT_Q2K && down_fmt != FMT_Q3K) return 1;
    if ((sh_gu_fmt != FMT_IQ2 && sh_gu_fmt != FMT_Q5K) || (sh_down_fmt != down_fmt && sh_down_fmt != FMT_Q6K)) return 1;
    const int E = HIDDEN, H = MOE_INTER;
    // q8 of every token's x
    std::vector<int8_t> xq((size_t)T * E); std::vector<float> xd((size_t)T * E / 32);
    orc_quant_q8(x, (int64_t)T * E, xq.data(), xd.data());
    // per-expert token lists (stable by (t, k))
    int maxid = 0; for (int i = 0; i < T * KE; ++i) maxid = std::max(maxid, ids[i]);
    const int NE = maxid + 1;
    std::vector<int> cnt(NE), off(NE + 1), perm((size_t)T * KE);
    orc_permute(ids, T, KE, NE, cnt.data(), off.data(), perm.data());
    std::vector<float> yslot((size_t)T * KE * E, 0.0f);
    std::vector<float> g((size_t)T * KE * H), u((size_t)T * KE * H);
    std::vector<int8_t> hq((size_t)T * KE * H); std::vector<float> hd((size_t)T * KE * H / 32);
    for (int m = 0; m < NE; ++m) {
        if (cnt[m] == 0) continue;
        const int n = cnt[m];
        std::vector<const int8_t*> xqp(n); std::vector<const float*> xdp(n); std::vector<float*> gp(n), up(n);
        for (int i = 0; i < n; ++i) {
            const int s = perm[off[m] + i], t = s / KE;
            xqp[i] = xq.data() + (size_t)t * E; xdp[i] = xd.data() + (size_t)t * E / 32;
            gp[i] = g.data() + (size_t)s * H; up[i] = u.data() + (size_t)s * H;
        }
        iq2_matvec_multi(Wl->gate + m * Wl->gate_stride, H, E, xqp.data(), xdp.data(), n, gp.data());
        iq2_matvec_multi(Wl->up + m * Wl->up_stride, H, E, xqp.data(), xdp.data(), n, up.data());
        std::vector<const int8_t*> hqp(n); std::vector<const float*> hdp(n); std::vector<float*> yp(n);
        std::vector<std::vector<float>> ytmp(n, std::vector<float>(E)), hf(n, std::vector<float>(H));
        std::vector<const float*> hfp(n);
        for (int i = 0; i < n; ++i) {
            const int s = perm[off[m] + i];
            for (int j = 0; j < H; ++j) hf[i][j] = lk_swiglu(g[(size_t)s * H + j], u[(size_t)s * H + j]);
            orc_quant_q8(hf[i].data(), H, hq.data() + (size_t)s * H, hd.data() + (size_t)s * H / 32);
            hqp[i] = hq.data() + (size_t)s * H; hdp[i] = hd.data() + (size_t)s * H / 32; yp[i] = ytmp[i].data();
            hfp[i] = hf[i].data();
        }
        if (down_fmt != FMT_IQ2 && hq8) kq_matvec_multi(down_fmt, Wl->down + m * Wl->down_stride, E, H, hqp.data(), hdp.data(), n, yp.data());
        else if (down_fmt != FMT_IQ2) kq_matvec_float_multi(down_fmt, Wl->down + m * Wl->down_stride, E, H, hfp.data(), n, yp.data());
        else if (hq8) iq2_matvec_multi(Wl->down + m * Wl->down_stride, E, H, hqp.data(), hdp.data(), n, yp.data());
        else iq2_matvec_float_multi(Wl->down + m * Wl->down_stride, E, H, hfp.data(), n, yp.data());
        for (int i = 0; i < n; ++i) {
            const int s = perm[off[m] + i];
            for (int j = 0; j < E; ++j) yslot[(size_t)s * E + j] = w[s] * ytmp[i][j];
        }
    }
    // shared expert on every token
    std::vector<float> sh((size_t)T * E, 0.0f);
    if (Wl->sh_gate) {
        std::vector<const int8_t*> xqp(T); std::vector<const float*> xdp(T);
        std::vector<float> sg((size_t)T * H), su((size_t)T * H); std::vector<float*> sgp(T), sup(T), shp(T);
        for (int t = 0; t < T; ++t) {
            xqp[t] = xq.data() + (size_t)t * E; xdp[t] = xd.data() + (size_t)t * E / 32;
            sgp[t] = sg.data() + (size_t)t * H; sup[t] = su.data() + (size_t)t * H; shp[t] = sh.data() + (size_t)t * E;
        }
        if (sh_gu_fmt == FMT_Q5K) {
            kq_matvec_multi(FMT_Q5K, Wl->sh_gate, H, E, xqp.data(), xdp.data(), T, sgp.data());
            kq_matvec_multi(FMT_Q5K, Wl->sh_up, H, E, xqp.data(), xdp.data(), T, sup.data());
        } else {
            iq2_matvec_multi(Wl->sh_gate, H, E, xqp.data(), xdp.data(), T, sgp.data());
            iq2_matvec_multi(Wl->sh_up, H, E, xqp.data(), xdp.data(), T, sup.data());
        }
        std::vector<int8_t> shq((size_t)T * H); std::vector<float> shd((size_t)T * H / 32), shf((size_t)T * H);
        std::vector<const int8_t*> hqp(T); std::vector<const float*> hdp(T), hfp(T);
        for (int t = 0; t < T; ++t) {
            float* hv = shf.data() + (size_t)t * H;
            for (int j = 0; j < H; ++j) hv[j] = lk_swiglu(sg[(size_t)t * H + j], su[(size_t)t * H + j]);
            orc_quant_q8(hv, H, shq.data() + (size_t)t * H, shd.data() + (size_t)t * H / 32);
            hqp[t] = shq.data() + (size_t)t * H; hdp[t] = shd.data() + (size_t)t * H / 32; hfp[t] = hv;
        }
        if (sh_down_fmt != FMT_IQ2 && (hq8 || sh_gu_fmt != FMT_IQ2))
            kq_matvec_multi(sh_down_fmt, Wl->sh_down, E, H, hqp.data(), hdp.data(), T, shp.data());
        else if (sh_down_fmt != FMT_IQ2) kq_matvec_float_multi(sh_down_fmt, Wl->sh_down, E, H, hfp.data(), T, shp.data());
        else if (hq8 || sh_gu_fmt != FMT_IQ2) iq2_matvec_multi(Wl->sh_down, E, H, hqp.data(), hdp.data(), T, shp.data());
        else iq2_matvec_float_multi(Wl->sh_down, E, H, hfp.data(), T, shp.data());
    }
    // combine in fixed k order
    #pragma omp parallel for schedule(static)
    for (int t = 0; t < T; ++t)
        for (int j = 0; j < E; ++j) {
            double r = 0.0;
            for (int k = 0; k < KE; ++k) r += (double)yslot[((size_t)t * KE + k) * E + j];
            if (moe) moe[(size_t)t * E + j] = (float)r;
            if (h) h[(size_t)t * E + j] = (float)(r + (double)sh[(size_t)t * E + j] + (double)resid[(size_t)t * E + j]);
        }
    if (y_slot) memcpy(y_slot, yslot.data(), yslot.size() * 4);
    if (shared_out) memcpy(shared_out, sh.data(), sh.size() * 4);
    return 0;
}

int orc_moe_layer_fmt(const float* x, const float* resid, int T, const OrcLayerW* Wl, const int* ids, const float* w,
                      int KE, float* h, float* moe, float* y_slot, float* shared_out, int hq8, int down_fmt) {
    return orc_moe_layer_fmt2(x, resid, T, Wl, ids, w, KE, h, moe, y_slot, shared_out, hq8, down_fmt, FMT_IQ2, down_fmt);
}

int orc_moe_layer_ex(const float* x, const float* resid, int T, const OrcLayerW* Wl, const int* ids, const float* w,
                     int KE, float* h, float* moe, float* y_slot, float* shared_out, int hq8) {
    return orc_moe_layer_fmt(x, resid, T, Wl, ids, w, KE, h, moe, y_slot, shared_out, hq8, FMT_IQ2);
}

int orc_moe_layer(const float* x, const float* resid, int T, const OrcLayerW* Wl, const int* ids, const float* w,
                  int KE, float* h, float* moe, float* y_slot, float* shared_out) {
    return orc_moe_layer_ex(x, resid, T, Wl, ids, w, KE, h, moe, y_slot, shared_out, 1);
}

// ------------------------------------------------------------------ ggml CPU numerics (an oracle mode)
// The reference's non-fused MoE path (src/server_core_fused.cpp:956-980) is a ggml graph: ggml_mul_mat_id for
// up, gate and down, ggml_swiglu_split, ggml_mul by the routing weights, the k slots added in order (:973),
// the shared expert by ggml_mul_mat (:974-975), then (moe + shared) + ffn_inp (:976).  On ggml's CPU backend
// the activations of IQ2_XXS and K-quant matrices are quantised to q8_K: one fp32 scale per 256 values.
// ggml is not vendored in the reference, so this mode restates ggml's published algorithm and is unpinned:
//   quantize_row_q8_K: per 256-block, max = the value of largest magnitude (the first on ties),
//     iscale = -127/max, q = min(127, round-half-even(iscale * x)), d = 1/iscale; an all-zero block gives
//     d = 0 and q = 0 (d is negative when max is positive: q * d still reconstructs x);
//   vec_dot_<fmt>_q8_K: exact integer sums of weight codes times q per sub-block, scaled in fp32 by the
//     block scales and d.  Here the same dot is evaluated in double from the dequantised weights (gguf-py
//     semantics, as above) and q * d: the ideal value of the q8_K scheme, which ggml's fp32 block
//     accumulation differs from by reassociation only;
//   silu(g) * u with g / (1 + exp(-g)) as lk_swiglu (ggml's expf and this file's lk_expf differ by an ulp
//     or so, far below the q8_K noise).
void orc_quant_q8_K(const float* x, int64_t n, int8_t* q, float* d) {
    for (int64_t b = 0; b < n / QK; ++b) {
        const float* xb = x + b * QK;
        int8_t* qb = q + b * QK;
        float amax = 0.0f, mx = 0.0f;
        for (int j = 0; j < QK; ++j) { const float a = fabsf(xb[j]); if (a > amax) { amax = a; mx = xb[j]; } }
        if (amax == 0.0f) { d[b] = 0.0f; memset(qb, 0, QK); continue; }
        const float iscale = -127.0f / mx;
        for (int j = 0; j < QK; ++j) qb[j] = (int8_t)std::min(127, (int)rintf(iscale * xb[j]));
        d[b] = 1.0f / iscale;
    }
}

// y[t][r] = W[r] . (q8_K of x[t]) for `ntok` rows given as codes xq[t][K] and scales xd[t][K/256]; W = rows x K
// in fmt (FMT_IQ2 or a K-quant), dequantised a row at a time
static void q8K_matvec_multi(int fmt, const uint8_t* W, int rows, int K, const int8_t* const* xq, const float* const* xd,
                             int ntok, float* const* y) {
    const int NB = K / QK, nb = fmt_block_bytes(fmt);
    #pragma omp parallel
    {
        std::vector<float> wr(K);
        std::vector<double> acc(ntok);
        #pragma omp for schedule(static)
        for (int r = 0; r < rows; ++r) {
            const uint8_t* row = W + (size_t)r * NB * nb;
            for (int b = 0; b < NB; ++b) {
                if (fmt == FMT_IQ2) iq2_deq_block(row + (size_t)b * nb, wr.data() + (size_t)b * QK);
                else kq_deq_block(fmt, row + (size_t)b * nb, wr.data() + (size_t)b * QK);
            }
            for (int t = 0; t < ntok; ++t) {
                double a = 0.0;
                for (int b = 0; b < NB; ++b) {
                    double s = 0.0;
                    for (int j = 0; j < QK; ++j) s += (double)wr[(size_t)b * QK + j] * (double)xq[t][(size_t)b * QK + j];
                    a += s * (double)xd[t][b];
                }
                acc[t] = a;
            }
            for (int t = 0; t < ntok; ++t) y[t][r] = (float)acc[t];
        }
    }
}

// one expert (gate/up in gu_fmt, down in dn_fmt) on n tokens: xq/xd are the tokens' q8_K codes and scales,
// y[i][HIDDEN] its outputs
static void q8K_expert(const uint8_t* gate, const uint8_t* up, const uint8_t* down, int gu_fmt, int dn_fmt,
                       const int8_t* const* xq, const float* const* xd, int n, float* const* y) {
    const int E = HIDDEN, H = MOE_INTER;
    std::vector<float> g((size_t)n * H), u((size_t)n * H), hf(H);
    std::vector<int8_t> hq((size_t)n * H); std::vector<float> hd((size_t)n * H / QK);
    std::vector<float*> gp(n), upp(n); std::vector<const int8_t*> hqp(n); std::vector<const float*> hdp(n);
    for (int i = 0; i < n; ++i) { gp[i] = g.data() + (size_t)i * H; upp[i] = u.data() + (size_t)i * H; }
    q8K_matvec_multi(gu_fmt, gate, H, E, xq, xd, n, gp.data());
    q8K_matvec_multi(gu_fmt, up, H, E, xq, xd, n, upp.data());
    for (int i = 0; i < n; ++i) {
        for (int j = 0; j < H; ++j) hf[j] = lk_swiglu(gp[i][j], upp[i][j]);
        orc_quant_q8_K(hf.data(), H, hq.data() + (size_t)i * H, hd.data() + (size_t)i * H / QK);
        hqp[i] = hq.data() + (size_t)i * H; hdp[i] = hd.data() + (size_t)i * H / QK;
    }
    q8K_matvec_multi(dn_fmt, down, E, H, hqp.data(), hdp.data(), n, y);
}

// The layer in ggml's CPU numerics: the arguments of orc_moe_layer_fmt2 (no slot outputs; hq8 does not apply:
// ggml always quantises h to q8_K).  moe = sum over k in order of fp32 w_k * y_k; h = (moe + shared) + resid.
int orc_moe_layer_ggml(const float* x, const float* resid, int T, const OrcLayerW* Wl, const int* ids, const float* w,
                       int KE, float* h, float* moe, float* shared_out, int down_fmt, int sh_gu_fmt, int sh_down_fmt) {
    if (down_fmt != FMT_IQ2 && down_fmt != FMT_Q2K && down_fmt != FMT_Q3K) return 1;
    if ((sh_gu_fmt != FMT_IQ2 && sh_gu_fmt != FMT_Q5K) || (sh_down_fmt != down_fmt && sh_down_fmt != FMT_Q6K)) return 1;
    const int E = HIDDEN;
    std::vector<int8_t> xq((size_t)T * E); std::vector<float> xd((size_t)T * E / QK);
    orc_quant_q8_K(x, (int64_t)T * E, xq.data(), xd.data());
    int maxid = 0; for (int i = 0; i < T * KE; ++i) maxid = std::max(maxid, ids[i]);
    const int NE = maxid + 1;
    std::vector<int> cnt(NE), off(NE + 1), perm((size_t)T * KE);
    orc_permute(ids, T, KE, NE, cnt.data(), off.data(), perm.data());
    std::vector<float> ys((size_t)T * KE * E);
    for (int m = 0; m < NE; ++m) {
        const int n = cnt[m];
        if (n == 0) continue;
        std::vector<const int8_t*> xqp(n); std::vector<const float*> xdp(n); std::vector<float*> yp(n);
        for (int i = 0; i < n; ++i) {
            const int s = perm[off[m] + i], t = s / KE;
            xqp[i] = xq.data() + (size_t)t * E; xdp[i] = xd.data() + (size_t)t * E / QK; yp[i] = ys.data() + (size_t)s * E;
        }
        q8K_expert(Wl->gate + m * Wl->gate_stride, Wl->up + m * Wl->up_stride, Wl->down + m * Wl->down_stride, FMT_IQ2,
                   down_fmt, xqp.data(), xdp.data(), n, yp.data());
    }
    std::vector<float> sh((size_t)T * E, 0.0f);
    if (Wl->sh_gate) {
        std::vector<const int8_t*> xqp(T); std::vector<const float*> xdp(T); std::vector<float*> yp(T);
        for (int t = 0; t < T; ++t) { xqp[t] = xq.data() + (size_t)t * E; xdp[t] = xd.data() + (size_t)t * E / QK; yp[t] = sh.data() + (size_t)t * E; }
        q8K_expert(Wl->sh_gate, Wl->sh_up, Wl->sh_down, sh_gu_fmt, sh_down_fmt, xqp.data(), xdp.data(), T, yp.data());
    }
    for (int t = 0; t < T; ++t)
        for (int j = 0; j < E; ++j) {
            float r = w[(size_t)t * KE] * ys[(size_t)t * KE * E + j];
            for (int k = 1; k < KE; ++k) r += w[(size_t)t * KE + k] * ys[((size_t)t * KE + k) * E + j];
            if (moe) moe[(size_t)t * E + j] = r;
            if (h) h[(size_t)t * E + j] = (r + sh[(size_t)t * E + j]) + resid[(size_t)t * E + j];
        }
    if (shared_out) memcpy(shared_out, sh.data(), sh.size() * 4);
    return 0;
}

}  // extern "C"

