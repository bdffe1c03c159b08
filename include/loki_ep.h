/* loki_ep.h -- expert-parallel MoE layer: 256 routed experts sharded over n_ranks GPUs of one node.
 *
 * No counterpart in the reference: its fused_layer.h drives one GPU and streams experts from NVMe
 * (src/moe_stream_buffer.h).  Here every rank keeps its shard (experts [r*E, (r+1)*E), E = 256/n_ranks)
 * resident in HBM, tokens stay on their home rank, and two all-to-all exchanges (done by the caller,
 * e.g. NCCL through torch.distributed) move rows to the experts and partial sums back:
 *
 *   home:   lk_moe_route -> lk_ep_pack -> send rows (every token also to its own rank)
 *   all-to-all #1 (rows)
 *   expert: lk_ep_experts(received rows) -> routed partial sums; the rows from this rank itself also get
 *           the shared expert in the same launches (a shared-expert-only stage is too small to fill a GPU)
 *   all-to-all #2 (partial sums, the transpose of #1)
 *   home:   lk_ep_combine -> h = resid + shared + sum of partials, moe = sum of partials
 *
 * A row is LK_EP_ROW_BYTES: a 64-byte header (int32 sel[8]: the expert id local to the receiving rank or
 * -1, float w[8]: routing weights), then the token's activations as their q8 per 32 -- int8 codes [7168] at
 * LK_EP_ROW_Q_OFF and fp32 scales [224] at LK_EP_ROW_D_OFF, the same quantisation the expert kernels apply
 * (d = amax/32-group / 127, round half even), so the experts compute exactly what they would from fp32 rows,
 * in 8 128 bytes instead of 28 736.  Rows for rank d form block
 * d of the send buffer, tokens ascending; block d starts at row d*cap (fixed capacity, cap >= T: no count
 * exchange needed, CUDA-graph friendly) or, with cap == 0, right after block d-1 (compact; the caller
 * exchanges send_counts first to size the transfer).  Unused rows of a fixed-capacity block have all sel
 * -1 and produce zero partial sums.  All pointers are device pointers; all calls are asynchronous on
 * `stream`.  Returns LK_OK or an LK_ERR_* code (loki_moe.h). */
#ifndef LOKI_EP_H
#define LOKI_EP_H
#include "loki_moe.h"

#ifdef __cplusplus
extern "C" {
#endif

#define LK_EP_ROW_HDR_BYTES 64
#define LK_EP_ROW_Q_OFF 64
#define LK_EP_ROW_D_OFF (64 + 7168)
#define LK_EP_ROW_BYTES (64 + 7168 + 7168 / 32 * 4)
#define LK_EP_MAX_RANKS 8

/* home side: sel/w [T][keep] (global expert ids, from lk_moe_route) and x [T][7168] -> send rows,
 * send_counts [n_ranks] (rows per destination) and row_map [T][n_ranks] (the send-buffer row of (t, d),
 * or -1).  self_rank >= 0: every token gets a row in that rank's block even without routed entries there
 * (its shared expert runs on it); -1: rows only where a token has entries.  keep <= 8, n_ranks in 1..8
 * dividing 256.  Ids outside [0, 256) set the context-free error word `err` (a device int, may be null)
 * and are dropped. */
LK_API int lk_ep_pack(const int* sel, const float* w, const float* x, int T, int keep, int n_ranks, int self_rank,
                      int cap, void* send_rows, int* send_counts, int* row_map, int* err, lk_stream_t stream);

/* expert side: R received rows -> out [R][7168] fp32, row r = sum over its entries of w * expert(x) in
 * entry order (the partial sum of the routed experts this rank owns); shared_out [shared_rows][7168] =
 * shared(x) of the rows [shared_row0, shared_row0 + shared_rows) (this rank's own tokens; 0 rows: none,
 * shared_out may be null).  ctx: a context with n_experts = the shard size, max_tokens >= R and
 * with_shared = 1 when shared_rows > 0; W: the shard's arenas (expert ids local) and shared expert. */
LK_API int lk_ep_experts(LkMoeCtx* ctx, const LkMoeWeights* W, const void* recv_rows, int R, int keep,
                         int shared_row0, int shared_rows, float* out, float* shared_out, lk_stream_t stream);

/* home side, when the shared expert is not folded into lk_ep_experts: h_partial [T][7168] = resid +
 * shared(x) of the home tokens.  ctx: a context with with_shared = 1 (W->sh_* set). */
LK_API int lk_ep_shared(LkMoeCtx* ctx, const LkMoeWeights* W, const float* x, const float* resid, int T,
                        float* h_partial, lk_stream_t stream);

/* home side, after the return exchange: ret rows in send-buffer order -> h = h_partial (+ shared, when
 * given) + sum_d ret and moe = sum_d ret (d ascending) for each of the T tokens; h_partial / h may be null
 * (then h is not written). */
LK_API int lk_ep_combine(const float* ret, const int* row_map, int T, int n_ranks, const float* h_partial,
                         const float* shared, float* h, float* moe, lk_stream_t stream);

/* the exchange: an NCCL communicator over the n_ranks GPUs (libnccl.so.2 bound at run time) and the
 * all-to-all of byte blocks.  lk_ep_comm_id (one rank) makes the LK_EP_COMM_ID_BYTES id every rank passes
 * to lk_ep_comm_create (collective: all ranks call it).  lk_ep_all_to_all sends block d of `send` (offset
 * send_off[d], send_bytes[d] bytes) to rank d and receives block s of `recv` from rank s (recv_off[s],
 * recv_bytes[s]); the offset / byte arrays are host arrays of n_ranks entries, or all null for equal blocks
 * of block_bytes at d * block_bytes.  Stream-ordered and CUDA-graph capturable; every rank must call it
 * with matching sizes. */
#define LK_EP_COMM_ID_BYTES 128
typedef struct LkEpComm LkEpComm;
LK_API int lk_ep_comm_id(void* id_out);
LK_API int lk_ep_comm_create(const void* id, int n_ranks, int rank, int device, LkEpComm** out);
LK_API void lk_ep_comm_destroy(LkEpComm* comm);
LK_API int lk_ep_all_to_all(LkEpComm* comm, const void* send, void* recv, const int64_t* send_off,
                            const int64_t* send_bytes, const int64_t* recv_off, const int64_t* recv_bytes,
                            int64_t block_bytes, lk_stream_t stream);

/* the peer-memory exchange for fixed-capacity (decode) layers: every rank owns a mailbox in its HBM (rows
 * received from each rank, partial sums returned by each owner, flags), exported by CUDA IPC and mapped by
 * every peer; senders store over NVLink and publish a flag, receivers poll their local flags with a
 * bounded wait (a timeout sets `err`).  Setup: lk_ep_mailbox_create on every rank (cap = the largest
 * per-rank token count, <= 64) gives an IPC handle; gather all n_ranks handles (LK_EP_IPC_HANDLE_BYTES
 * each, rank order) and pass them to lk_ep_mailbox_connect.  Per layer, on one stream:
 *   lk_ep_p2p_dispatch (rows into the owners' mailboxes; every token also to itself; row_map)
 *   lk_ep_p2p_rows (wait for all ranks' rows; *rows = n_ranks*cap rows in fixed-capacity order)
 *   lk_ep_experts(rows, n_ranks*cap, ..., own rows rank*cap .. +T, partial, shared)
 *   lk_ep_p2p_return(partial)  (each block of cap partial sums to its home rank)
 *   lk_ep_p2p_combine (wait for all returns; h = resid + shared + sum, moe = sum)
 * (with one token, lk_ep_p2p_route_dispatch does the routing and the dispatch in the router's launch), or, for
 * the single-token expert path (n_ranks*cap rows below the context's mma threshold and at most 64, an
 * IQ2_XXS or no shared expert: decode), the direct return:
 *   lk_ep_p2p_experts(mb, ctx, W, keep, T, shared, err)  (the rows wait fused with the slot tables, the expert
 *     kernels reading the rows' q8 codes, the down kernel storing each entry's weighted row straight into its
 *     home rank's mailbox; LK_ERR_UNSUPPORTED outside that path)
 *   lk_ep_p2p_combine_entries(mb, sel, keep, row_map, ...)  (publish this rank's return flags, wait for all
 *     owners; h = resid + shared + the entries summed in k order, moe = that sum: the single-GPU combine's
 *     order).  A rank with T = 0 calls no combine: its lk_ep_p2p_experts publishes the flags itself.
 * All kernels are capturable; the flags carry an epoch that advances per layer on the device. */
#define LK_EP_IPC_HANDLE_BYTES 64
typedef struct LkEpMailbox LkEpMailbox;
LK_API int lk_ep_mailbox_create(int n_ranks, int rank, int cap, int device, LkEpMailbox** out, void* ipc_handle_out);
LK_API int lk_ep_mailbox_connect(LkEpMailbox* mb, const void* handles);
LK_API void lk_ep_mailbox_destroy(LkEpMailbox* mb);
LK_API int lk_ep_p2p_dispatch(LkEpMailbox* mb, const int* sel, const float* w, const float* x, int T, int keep,
                              int* row_map, int* err, lk_stream_t stream);
LK_API int lk_ep_p2p_rows(LkEpMailbox* mb, const void** rows, int* err, lk_stream_t stream);
LK_API int lk_ep_p2p_return(LkEpMailbox* mb, const float* partial, lk_stream_t stream);
LK_API int lk_ep_p2p_combine(LkEpMailbox* mb, const int* row_map, int T, const float* resid, const float* shared,
                             float* h, float* moe, int* err, lk_stream_t stream);
/* no reference counterpart (the reference runs on one GPU): lk_ep_p2p_rows + lk_ep_experts + lk_ep_p2p_return
 * with the rows wait, the header unpack and the slot building in one kernel, and the return stored by the
 * down kernel itself (one row per routed entry, in the home mailbox); shared [T][7168] receives the shared
 * expert of this rank's own T rows.  Pair it with lk_ep_p2p_combine_entries. */
LK_API int lk_ep_p2p_experts(LkEpMailbox* mb, LkMoeCtx* ctx, const LkMoeWeights* W, int keep, int T, float* shared,
                             int* err, lk_stream_t stream);
/* no reference counterpart: lk_moe_route + lk_ep_p2p_dispatch for one token (T == 1, else LK_ERR_UNSUPPORTED)
 * as one launch -- the router's last CTA, after its top-k, stores the token's row (the router's q8 of x) into
 * every rank's mailbox and publishes the flags.  ctx: the home (256-expert) context; sel/w [1][keep] and
 * row_map [1][n_ranks] out, as the two calls give them. */
LK_API int lk_ep_p2p_route_dispatch(LkEpMailbox* mb, LkMoeCtx* ctx, const LkMoeWeights* W, const float* x, int T,
                                    const float* logits_override, int* sel, float* w, int* row_map, int* err,
                                    lk_stream_t stream);
/* no reference counterpart: the home combine of lk_ep_p2p_experts' direct return; sel [T][keep] the routing
 * passed to lk_ep_p2p_dispatch (global ids, negative = absent), row_map its output */
LK_API int lk_ep_p2p_combine_entries(LkEpMailbox* mb, const int* sel, int keep, const int* row_map, int T,
                                     const float* resid, const float* shared, float* h, float* moe, int* err,
                                     lk_stream_t stream);

#ifdef __cplusplus
}
#endif
#endif
