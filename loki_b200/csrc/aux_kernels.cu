// aux_kernels.cu -- small kernels around the expert stage: the combine (h = resid + shared + sum_k y;
// reference moe_combine / wide_finish, src/fused_layer.cu:358-373) and the seeded IQ2_XXS generator.
#include "moe_internal.h"
#include "moe_device.cuh"

namespace lk {

// ------------------------------------------------------------------ combine
__global__ void __launch_bounds__(64) k_combine(CombineParams p) {
    pdl_trigger();
    pdl_wait();
    const int i = blockIdx.x * blockDim.x + threadIdx.x;       // float4 index over T x HIDDEN
    const int per = HIDDEN / 4;
    if (i >= p.T * per) return;
    const int t = i / per, c = i % per;
    // every load is issued before any sum (one memory round trip); the sums keep entry order
    float4 v[MAX_TOPK];
    bool use[MAX_TOPK];
    const float4 zero = make_float4(0.f, 0.f, 0.f, 0.f);
    #pragma unroll
    for (int k = 0; k < MAX_TOPK; ++k) {
        use[k] = k < p.keep && !(p.sel && p.sel[t * p.keep + k] < 0);
        v[k] = k < p.keep ? ((const float4*)(p.y + ((size_t)t * p.keep + k) * HIDDEN))[c] : zero;
    }
    const int nsh = p.sh_n < 0 ? 0 : (p.sh_n > 0 ? p.sh_n : p.T), j = t - p.sh_t0;
    const bool in_sh = p.with_shared && j >= 0 && j < nsh;
    const bool has_sh = p.h && in_sh;
    const float4 hr = p.h && p.resid ? ((const float4*)(p.resid + (size_t)t * p.ld_out))[c] : zero;
    const float4 hs = in_sh && (p.h || p.shared_out) ? ((const float4*)(p.y + ((size_t)p.T * p.keep + j) * HIDDEN))[c] : zero;
    if (in_sh && p.shared_out) ((float4*)(p.shared_out + (size_t)j * HIDDEN))[c] = hs;
    const float4 he = p.h && p.shared ? ((const float4*)(p.shared + (size_t)t * HIDDEN))[c] : zero;
    float4 r = zero;
    #pragma unroll
    for (int k = 0; k < MAX_TOPK; ++k)
        if (use[k]) { r.x += v[k].x; r.y += v[k].y; r.z += v[k].z; r.w += v[k].w; }
    if (i == 0 && p.err2) *p.err2 = *p.err;          // every earlier kernel's error (they have completed)
    if (p.moe) ((float4*)(p.moe + (size_t)t * p.ld_out))[c] = r;
    if (p.moe2) ((float4*)(p.moe2 + (size_t)t * p.ld_out))[c] = r;
    if (!p.h) return;
    float4 h = hr;
    if (has_sh) { h.x += hs.x; h.y += hs.y; h.z += hs.z; h.w += hs.w; }
    if (p.shared) { h.x += he.x; h.y += he.y; h.z += he.z; h.w += he.w; }
    h.x += r.x; h.y += r.y; h.z += r.z; h.w += r.w;
    ((float4*)(p.h + (size_t)t * p.ld_out))[c] = h;
    if (p.h2) ((float4*)(p.h2 + (size_t)t * p.ld_out))[c] = h;
}

void launch_combine(const CombineParams& p, cudaStream_t st) {
    const int n = p.T * (HIDDEN / 4);
    launch_pdl(k_combine, dim3((n + 63) / 64), dim3(64), 0, st, p);
}

// ------------------------------------------------------------------ seeded weight generation
// one CTA = 64 consecutive blocks of one expert matrix, staged in shared memory, written as 16-byte words
__global__ void __launch_bounds__(64) k_gen_iq2(uint8_t* dst, uint64_t seed, int layer, int matrix, int expert0,
                                                int rows, int K, int64_t stride, int fmt) {
    __shared__ __align__(16) uint8_t buf[64 * BLK_Q6K];        // the largest block (210 B)
    const int e = expert0 + blockIdx.y;
    const int nbytes = fmt_block_bytes(fmt);
    const uint64_t key = iq2_gen_key(seed, (uint32_t)layer, (uint32_t)matrix, (uint32_t)e);
    const int64_t nblk = (int64_t)rows * (K / QK);
    const int64_t b0 = (int64_t)blockIdx.x * 64;
    const int64_t b = b0 + threadIdx.x;
    if (b < nblk) {
        if (fmt == FMT_IQ2) iq2_gen_block(key, (uint64_t)b, buf + threadIdx.x * BLK_IQ2);
        else kq_gen_block(fmt, key, (uint64_t)b, buf + threadIdx.x * nbytes);
    }
    __syncthreads();
    uint8_t* out = dst + (size_t)blockIdx.y * stride + (size_t)b0 * nbytes;
    const int nb = (int)(nblk - b0 < 64 ? nblk - b0 : 64);
    const int bytes = nb * nbytes;
    if (((uintptr_t)out & 15) == 0 && (bytes & 15) == 0) {
        for (int i = threadIdx.x; i < bytes / 16; i += 64) ((uint4*)out)[i] = ((const uint4*)buf)[i];
    } else {
        for (int i = threadIdx.x; i < bytes; i += 64) out[i] = buf[i];
    }
}

void launch_gen_iq2(uint8_t* dst, uint64_t seed, int layer, int matrix, int expert0, int n_exp, int rows, int K,
                    int64_t stride, cudaStream_t st) {
    const int64_t nblk = (int64_t)rows * (K / QK);
    dim3 grid((unsigned)((nblk + 63) / 64), (unsigned)n_exp);
    k_gen_iq2<<<grid, 64, 0, st>>>(dst, seed, layer, matrix, expert0, rows, K, stride, FMT_IQ2);
}

void launch_gen_weights(int fmt, uint8_t* dst, uint64_t seed, int layer, int matrix, int expert0, int n_exp, int rows, int K,
                        int64_t stride, cudaStream_t st) {
    const int64_t nblk = (int64_t)rows * (K / QK);
    dim3 grid((unsigned)((nblk + 63) / 64), (unsigned)n_exp);
    k_gen_iq2<<<grid, 64, 0, st>>>(dst, seed, layer, matrix, expert0, rows, K, stride, fmt);
}

int num_sms(int device) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device);
    return n;
}

}  // namespace lk
