// moe_internal.h -- kernel parameter blocks and launchers shared by the library's translation units.
#pragma once
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <stdint.h>
#include "moe_format.h"

namespace lk {

constexpr int SHARED_SLOT = -1;      // slot_expert value of the shared expert
constexpr int MAX_NT = 8;            // tokens per work slot of the grouped matvecs
constexpr int GEMM_NT = 128;         // tokens per work slot of the tensor-core GEMMs (prefill)
constexpr int MM_NT = 16;            // tokens per work slot of the register-fed mma.sync products (mid-size T)

// ---- router
// optional, T == 1 (expert-parallel decode over the peer mailboxes, ep_p2p.cu): after the top-k, the router's last
// CTA sends the token's row to every rank (include/loki_ep.h row format, the q8 of x from xq/xd), writes
// row_map [n_ranks] and publishes every rank's rows flag; n_ranks = 0: no send
struct EpSendParams {
    uint8_t* mb[8];                         // every rank's mailbox base, as mapped in this process
    int n_ranks, self, cap;
    int* row_map;
};

struct RouterParams {
    const float* x; int T; int ld_x;        // activations [T][HIDDEN], row stride ld_x floats
    const void* W; int w_f16;               // router weights [n_experts][HIDDEN], fp32 or fp16
    const float* logits_override;           // optional [T][n_experts]: selection from these logits instead
    const float* bias;                      // e_score_correction bias [n_experts]
    float* logits;                          // [T][n_experts] out (the GEMV result)
    float* probs;                           // [T][n_experts] out: sigmoid of the logits used for selection
    int* sel; float* w;                     // [T][keep] out
    int n_experts, topk, keep, renorm, n_group, topk_group; float scale;
    // optional slot table written directly for T == 1 (decode): keep routed slots + shared slot
    int* slot_expert; int* slot_tok; int* slot_out; float* slot_w; int* nslots; int with_shared;
    int* tile_count;                        // T zeroed counters (last-CTA-done top-k; one per token tile)
    // optional, T == 1: the q8 of x for the expert kernels -- CTA e < HIDDEN/32 writes group e: int8 values
    // xq, their negations xqn (HIDDEN bytes each) and the scale xd[e] (quant_q8_group, bit for bit)
    int8_t* xq; int8_t* xqn; float* xd;
    EpSendParams send;                      // optional, T == 1 (needs xq): the expert-parallel send
    int esplit;                             // set by launch_router: expert splits of the batch kernel
};
void launch_router(const RouterParams& p, cudaStream_t st);

// Programmatic dependent launch for the decode chain (router -> gate/up -> down -> combine -> next router):
// the kernel may start while its predecessor still runs.  Each such kernel only sets up shared memory (and
// reads never-written inputs such as weights) before griddepcontrol.wait, and triggers its own
// dependents once its CTAs are running, so a dependent grid is only scheduled after every CTA of its
// predecessor is resident (no SM starvation).
template <typename P>
inline cudaError_t launch_pdl(void (*kernel)(P), dim3 grid, dim3 block, size_t smem, cudaStream_t st, const P& params) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid; cfg.blockDim = block; cfg.dynamicSmemBytes = smem; cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr; cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, params);
}
// the same for kernels with several parameters
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl_n(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args... args) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid; cfg.blockDim = block; cfg.dynamicSmemBytes = smem; cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr; cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

// ---- dispatch: per-expert stable token lists and the work-slot table of the grouped matvecs
struct SlotParams {
    const int* sel; const float* w; int T; int keep;   // [T][keep]; negative ids are absent entries (skipped)
    int n_experts; int nt;                              // tokens per slot (<= MAX_NT)
    int with_shared;
    int* counts; int* offsets; int* perm;               // [n_experts], [n_experts+1], [T*keep]
    int* slot_expert; int* slot_tok; int* slot_out; float* slot_w; int* nslots;   // slot tables
    int max_slots;
    int* err;                                           // device error word (bad expert ids)
    // shared-expert slots (with_shared) cover tokens [sh_t0, sh_t0 + sh_n) -- sh_n = 0: all T tokens from 0,
    // sh_n < 0: none; their entry rows are T*keep + (t - sh_t0)
    int sh_t0, sh_n;
};
void launch_build_slots(const SlotParams& p, cudaStream_t st);
int max_slots_for(int T, int keep, int n_experts, int nt, int with_shared);

// ---- expert-parallel single-token stage (ep_p2p.cu, ep_device.cuh)
// the direct return's destinations: entry (row i / keep, k = i % keep) of received row (source s = row / cap,
// r = row % cap) goes to ret[s] + ((self * cap + r) * MAX_TOPK + k) * HIDDEN -- its row in the home rank's
// mailbox -- and shared slot j to shared_out + j * HIDDEN; ydst [max_slots] receives the row pointers
struct EpYDst {
    float* ret[8];
    int self, cap;
    float* shared_out;
    float** ydst;
};
// the rows wait + slot tables run by the single-token gate/up kernel itself (every CTA): mb this rank's mailbox,
// sel/w [n_ranks*cap][keep] out, sp the slot tables, yd the destinations (yd.ydst null: none); mb null: none
struct EpWait {
    uint8_t* mb;
    int n_ranks, cap, keep, n_experts;
    int* sel; float* w;
    SlotParams sp;
    EpYDst yd;
    int* err;
};

// ---- grouped IQ2_XXS matvecs on work slots
struct ExpertParams {
    // arenas: routed expert e's matrices at base + e*stride; the shared expert's at sh_*
    const uint8_t* gate; const uint8_t* up; const uint8_t* down;
    int64_t gate_stride, up_stride, down_stride;
    const uint8_t* sh_gate; const uint8_t* sh_up; const uint8_t* sh_down;
    const float* x; int ld_x;                         // activations [T][HIDDEN] (fp32; quantised to q8 in-kernel)
    const int* slot_expert; const int* slot_tok; const int* slot_out; const float* slot_w; const int* nslots;
    const int8_t* xq; const int8_t* xqn; const float* xd;   // optional: token 0's q8 activations from the router
    // optional: the activations as expert-parallel rows (include/loki_ep.h): token t's q8 codes and scales read
    // from row t (the single-token gate/up only; x is then not read)
    const uint8_t* xrows;
    int8_t* hq; float* hd;                            // SwiGLU output q8: [rows][MOE_INTER], scales [rows][MOE_INTER/32]
    float* y;                                         // weighted expert outputs [rows][HIDDEN]
    // optional (single-token downs): slot s writes its weighted output row to ydst[s] instead of y row
    // slot_out[s] (the expert-parallel direct return: rows in the home rank's mailbox, over NVLink)
    float* const* ydst;
    EpWait epw;                                       // optional (single-token gate/up): the rows wait + slot tables
    int* err;
    int down_fmt;                                     // FMT_IQ2 (default, 0 reads as IQ2), FMT_Q2K or FMT_Q3K: every down matrix
    // shared-only launches of launch_down1_kq (slot_expert == null): sh_count single-token slots, slot j
    // reading sh_down and the q8 h of hq/hd row sh_row0 + j into y row sh_row0 + j (weight 1)
    int sh_count, sh_row0;
};
void launch_gate_up(const ExpertParams& p, int nt, int grid, cudaStream_t st);
void launch_down(const ExpertParams& p, int nt, int grid, cudaStream_t st);
// single-token down projection of K-quant (Q2_K / Q3_K) experts (expert_kq.cu)
void launch_down1_kq(const ExpertParams& p, int grid, cudaStream_t st);

// the real model's shared expert (Q5_K gate/up, Q6_K down; shared_kq.cu) of tokens [t0, t0 + n) of x as its
// own launches: gate/up rows into gu (fp32 [n][2][MOE_INTER]), SwiGLU q8 into hq/hd rows row0 + j, the down
// into y rows row0 + j (weight 1).  pair: n * 64 zeroed counters (left zeroed)
struct SharedKqParams {
    const uint8_t* gate; const uint8_t* up; const uint8_t* down;
    const float* x; int ld_x;
    int t0, n, row0;
    const int8_t* xq; const float* xd;                // optional: token 0's q8 x from the router
    float* gu; int8_t* hq; float* hd; int* pair; float* y; int* err;
};
void launch_shared_kq(const SharedKqParams& p, int grid, cudaStream_t st);

// the same shared expert for many tokens as dense tcgen05 GEMMs (shared_gemm.cu): its three matrices
// dequantised (w16: SH_GEMM_W16_BYTES; gate/up as fp16 hi/lo pairs, down fp16), the q8 of x as fp16 hi/lo
// token tiles (x16: 4 * HIDDEN bytes per padded token), gate/up with SwiGLU and the q8 of h as fp16 into h16
// (2 * MOE_INTER bytes per padded token), the down into y rows row0 + j.  Tokens are padded to
// sh_gemm_pad(n).  Returns 0, or 1 on a launch error.
constexpr size_t SH_GEMM_W16_BYTES = (size_t)2 * 2 * MOE_INTER * HIDDEN * 2 + (size_t)HIDDEN * MOE_INTER * 2;
struct SharedGemmParams {
    const uint8_t* gate; const uint8_t* up; const uint8_t* down;
    const float* x; int ld_x; int t0, n, row0;
    uint8_t* w16; uint8_t* x16; uint8_t* h16; float* y; int* err;
};
int sh_gemm_tile_tokens(int n);
inline int sh_gemm_pad(int n) { const int nt = sh_gemm_tile_tokens(n); return (n + nt - 1) / nt * nt; }
int launch_shared_gemm(const SharedGemmParams& p, cudaStream_t st);

// ---- combine: h = resid + shared + sum_k y[t*keep+k], moe = sum_k y[t*keep+k]
//      (shared = the y rows T*keep + t when with_shared, and/or the separate `shared` rows)
struct CombineParams {
    const float* y; const float* resid; int T; int keep; int with_shared;
    const float* shared;              // optional [T][HIDDEN] shared-expert output added to h
    float* h; float* moe; int ld_out;
    const int* sel;                   // optional [T][keep]: entries with a negative id are not summed
    int sh_t0, sh_n;                  // shared-expert rows as in SlotParams; resid may be null (zero)
    float* shared_out;                // optional: the shared expert's output of rows [sh_t0, +sh_n) -> row j here
    // optional second destinations of h and moe (ld_out as well): page-locked host memory the kernel stores into
    // directly, so no device-to-host copy follows; err2 (with err): a copy of the device error word, by one thread
    float* h2; float* moe2; const int* err; int* err2;
};
void launch_combine(const CombineParams& p, cudaStream_t st);

// ---- tensor-core grouped GEMMs (prefill / batch): slots of up to GEMM_NT tokens
struct GemmParams {
    const uint8_t* gate; const uint8_t* up; const uint8_t* down;
    int64_t gate_stride, up_stride, down_stride;
    const uint8_t* sh_gate; const uint8_t* sh_up; const uint8_t* sh_down;
    const float* x; int ld_x; int T;                  // activations [T][HIDDEN] fp32
    const int* slot_expert; const int* slot_tok; const int* slot_out; const float* slot_w; const int* nslots;  // [slot][GEMM_NT]
    int max_slots;
    int* slot_cnt;                                    // [max_slots] tokens per slot (written by the gate/up B-tile pre-pass)
    __half* bt;                                       // gate/up activation tiles [max_slots][HIDDEN/128][2 halves][hi, lo rows][128]
    __half* ht;                                       // down B tiles (fp16 of the q8 h) [max_slots][MOE_INTER/128][N x 128]
    float* y;                                         // [rows][HIDDEN] weighted expert outputs
    int* err;
    __half* hb;                                       // optional: the SwiGLU output as fp16 rows [entry][MOE_INTER]
                                                      //   instead of the down B tiles (the mma.sync downs read them)
};
// the IQ2_XXS down GEMM (prefill_gemm.cu), reading the B tiles ht that launch_gate_up_q8 wrote (hb null)
void launch_prefill_gemm_down(const GemmParams& p, int grid, cudaStream_t st);
size_t down_tile_halfs(int max_slots);                // size of ht in halfs
// the gate/up + SwiGLU phase with the reference's q8 numerics (gate_up_q8.cu): exact products, h re-quantised
// to q8 per 32; writes fp16(q*d) as the down GEMM's B tiles (ht) or, with hb set, as fp16 rows [entry][MOE_INTER].
// bt must hold gate_q8_tile_halfs(max_slots) halfs (hi and lo activation rows per token half).
void launch_gate_up_q8(const GemmParams& p, int grid, cudaStream_t st);
size_t gate_q8_tile_halfs(int max_slots);

// ---- register-fed mma.sync downs (slot_mma.cu IQ2_XXS, kq_mma.cu Q2_K / Q3_K): slots of up to MM_NT tokens
//      reading the fp16 q8 SwiGLU rows that the q8 gate/up wrote
struct MmaParams {
    const uint8_t* down; int64_t down_stride; const uint8_t* sh_down;
    const int* slot_expert; const int* slot_tok; const int* slot_out; const float* slot_w; const int* nslots;  // [slot][MM_NT]
    int max_slots;
    int* slot_cnt;                                    // [max_slots] tokens per slot (slot_mma's prep pass; null: counted in-kernel)
    __half* hb;                                       // [rows][MOE_INTER] fp16 SwiGLU output
    float* y;                                         // [rows][HIDDEN] weighted expert outputs
    int* err;
};
// the IQ2_XXS down on MM_NT slots (its prep pass writes slot_cnt)
void launch_slot_mma_down(const MmaParams& p, int nsm, cudaStream_t st);
// the Q2_K / Q3_K down on MM_NT slots (kq_mma.cu)
void launch_kq_mma_down(const MmaParams& p, int down_fmt, int nsm, cudaStream_t st);

// ---- seeded IQ2_XXS weight generation (moe_format.h generator) for n_experts consecutive experts
void launch_gen_iq2(uint8_t* dst, uint64_t seed, int layer, int matrix, int expert0, int n_exp, int rows, int K,
                    int64_t stride, cudaStream_t st);
// ---- the same for any down format (FMT_IQ2, or the K-quants' kq_gen_block)
void launch_gen_weights(int fmt, uint8_t* dst, uint64_t seed, int layer, int matrix, int expert0, int n_exp, int rows, int K,
                        int64_t stride, cudaStream_t st);

// ---- expert-parallel row headers -> sel/w [R][keep], and (x non-null) the rows' q8 activations -> fp32
void launch_ep_unpack(const void* recv, int R, int keep, int* sel, float* w, float* x, cudaStream_t st);   // x: [R][HIDDEN]
// the same headers -> sel/w, plus the single-token slot tables of sp (slot_*, nslots, max_slots, with_shared,
// sh_t0, sh_n, err) built directly: one slot per live entry, then the shared expert's slots
struct SlotParams;
void launch_ep_slots(const void* recv, int R, int keep, int n_experts, int* sel, float* w, const SlotParams& sp, cudaStream_t st);
}  // namespace lk
struct LkEpMailbox;
namespace lk {
// the peer exchange's fused stage (ep_p2p.cu) for lk_ep_p2p_experts: the rows wait + the single-token slot tables
// of the received rows (*rows: the mailbox's rows)
int p2p_rows_count(const LkEpMailbox* m);
int p2p_rank(const LkEpMailbox* m);
int p2p_cap(const LkEpMailbox* m);
// the single-token gate/up's rows wait + slot tables for mailbox m (ydst with shared_out: the direct return's
// destinations); *rows: the received rows.  LK_ERR_ARG: not connected
int p2p_rows_wait(LkEpMailbox* m, int keep, int n_experts, int* sel, float* w, const SlotParams& sp, int* err,
                  float** ydst, float* shared_out, EpWait* out, const uint8_t** rows);
bool p2p_direct_ok(const LkEpMailbox* m);
// the direct return's flags: once the down kernel (the previous launch) has stored every entry row, this layer's
// epoch + 1 into every home rank's return flag of this rank, and the local epoch advances to it (after
// p2p_rows_wait, whose waits read the epoch unadvanced)
int p2p_ret_flags(LkEpMailbox* m, cudaStream_t st);
// the router's send parameters for mailbox m (row_map [n_ranks] out); false: not connected
bool p2p_send_params(const LkEpMailbox* m, int* row_map, EpSendParams* out);

// ---- expert-parallel row plan only: counts [n_ranks], row_map [T][n_ranks] (and, with `send`, the
//      headers of unused fixed-capacity rows)
int ep_plan(const int* sel, int T, int keep, int n_ranks, int self_rank, int cap, int* counts, int* row_map, uint8_t* send,
            int* err, cudaStream_t st);

int num_sms(int device);

}  // namespace lk
