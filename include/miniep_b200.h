/*
 * libminiep_b200 — expert-parallel MoE layer for B200 (sm_100a), C ABI.
 *
 * Drop-in compute path behind mini-EP's MoE-backend contract
 * (kanwarpal-brar/mini-ep, miniep/ep.py and miniep/modeling.py). The reference
 * is Python; its FFI for this path would be ctypes, so every entry point takes
 * plain pointers and sizes only:
 *   - tensor arguments are DEVICE pointers (contiguous, row-major) unless the
 *     comment says "host";
 *   - `stream` is a cudaStream_t passed as void*; all GPU work is enqueued on
 *     it and nothing synchronises unless stated;
 *   - dtype codes: MEP_F32 (fp32 everywhere) or MEP_BF16 (bf16 activations,
 *     weights, gates; fp32 accumulation);
 *   - every function returns MEP_OK (0) or an error code; mep_last_error()
 *     gives the message. Device-side failures (a routing index outside
 *     [0, E), a receive buffer overflow, a peer that never signalled) are
 *     recorded in a host-mapped error word and reported by mep_check() after
 *     the caller has synchronised the stream.
 *
 * One context per rank (one process per GPU). All ranks must issue the same
 * sequence of forward calls (lockstep), exactly like the reference's
 * collectives; a rank with no tokens still calls with n = 0.
 */
#ifndef MINIEP_B200_H_
#define MINIEP_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MEP_OK 0
#define MEP_ERR_INVALID 1   /* bad argument (shape, pointer, placement) */
#define MEP_ERR_CUDA 2      /* a CUDA runtime call failed */
#define MEP_ERR_DEVICE 3    /* the device error word is set (see mep_check) */
#define MEP_ERR_STATE 4     /* call out of order (e.g. placement not set) */

#define MEP_F32 0
#define MEP_BF16 1

#define MEP_IPC_HANDLE_BYTES 64

typedef struct mep_ctx mep_ctx;

/* Library version (major*10000 + minor*100 + patch). */
int mep_version(void);

/* Message for the last failed call on `ctx`; with ctx NULL, of the last failed
 * call that takes no context (mep_ctx_create, mep_dest_ranks_noalloc). */
const char* mep_last_error(const mep_ctx* ctx);

/*
 * Per-rank context: device buffers for the layer step, the placement tables,
 * the round-robin state and the routing statistics.
 *   replaces: Comm() + EPStats(L, E) + the per-layer EPMoEBackend state
 *             (miniep/ep.py:110-118, ep.py:164-173, ep.py:193-208,
 *              construction in miniep/worker.py:76-95)
 * max_tokens: largest token count per call on this rank.
 * recv_capacity_rows: receive-buffer rows (0 = worst case, every entry of
 *             every rank landing here plus per-expert padding).
 */
int mep_ctx_create(int rank, int world, int device, int num_layers, int num_experts, int topk,
                   int hidden, int inter, int64_t max_tokens, int dtype,
                   int64_t recv_capacity_rows, mep_ctx** out);
int mep_ctx_destroy(mep_ctx* ctx);

/*
 * Symmetric-memory set-up for world > 1: export this rank's buffer handle
 * (MEP_IPC_HANDLE_BYTES bytes, host) and open every peer's. Exchanging the
 * handles is the caller's job (the Python host uses torch.distributed).
 *   replaces: the gloo process group the reference's Comm runs on
 *             (miniep/worker.py:285, ep.py:114-118)
 */
int mep_ipc_handle(mep_ctx* ctx, void* handle_out);
int mep_ipc_open(mep_ctx* ctx, int peer, const void* handle);

/*
 * Placement of one layer: table (host, E x rmax, int64) holds the ranks of
 * expert e's replicas in table[e*rmax + j] for j < n_rep[e] (owner lists
 * sorted, distinct). The same table must be given on every rank.
 *   replaces: Placement._build_table / Placement(owners) (miniep/ep.py:27-45);
 *             the plan JSON (ep.py:54-65) is parsed by the host wrapper.
 */
int mep_set_placement(mep_ctx* ctx, int layer, const int64_t* table, const int64_t* n_rep,
                      int rmax);

/* Zero the per-(layer, expert) round-robin counters.
 *   replaces: Placement.reset_rr (miniep/ep.py:73-74) */
int mep_reset_rr(mep_ctx* ctx, void* stream);

/*
 * Destination rank of each of m expert ids under replica round-robin, updating
 * the round-robin state exactly as the reference does.
 *   replaces: Placement.dest_ranks (miniep/ep.py:76-96)
 * expert_ids: (m,) int64; dest_out: (m,) int64. m <= max_tokens * topk.
 */
int mep_dest_ranks(mep_ctx* ctx, int layer, const int64_t* expert_ids, int64_t m,
                   int64_t* dest_out, void* stream);

/*
 * Router: logits = x @ router_w^T in the model dtype, + bias (optional, (E,)
 * fp32, rounded to the model dtype), top-k (ties to the lower index), softmax
 * over the k logits in fp32, gates cast to the model dtype.
 *   replaces: Block.forward lines miniep/modeling.py:193-195
 * x: (n, H); router_w: (E, H); topk_idx_out: (n, k) int64;
 * topk_gate_out: (n, k) model dtype; logits_out: (n, E) fp32 or NULL.
 */
int mep_router_topk(mep_ctx* ctx, const void* x, const void* router_w, const float* bias,
                    int64_t n, int64_t* topk_idx_out, void* topk_gate_out, float* logits_out,
                    void* stream);

/*
 * One MoE layer step for this rank's n tokens: route (with replica
 * round-robin), exchange counts, dispatch rows to their expert owners, run the
 * grouped SwiGLU experts, return the outputs and combine them in slot order.
 * Updates route_counts[layer] and recv_tokens_per_layer[layer].
 *   replaces: EPMoEBackend.__call__ (miniep/ep.py:210-249), which is also
 *             LocalMoEBackend.__call__ (miniep/modeling.py:138-145) at world 1
 * x: (n, H), rows contiguous, starting on a 16-byte boundary; topk_idx: (n, k)
 * int64; topk_gate: (n, k) model dtype;
 * valid: (n,) uint8 or NULL (all valid); w_in: (n_local, 2I, H) and
 * w_out: (n_local, H, I) for this rank's experts of `layer` in increasing
 * expert order; out: (n, H).
 */
int mep_moe_forward(mep_ctx* ctx, int layer, const void* x, const int64_t* topk_idx,
                    const void* topk_gate, const uint8_t* valid, int64_t n, const void* w_in,
                    const void* w_out, int n_local, void* out, void* stream);

/*
 * Router + MoE layer step + residual: h_out = h + moe(x) * residual_multiplier.
 *   replaces: Block.forward lines miniep/modeling.py:192-197
 * topk_idx_out / topk_gate_out: (n, k) outputs (device scratch the caller owns).
 */
int mep_moe_block(mep_ctx* ctx, int layer, const void* h, const void* x, const void* router_w,
                  const float* bias, const uint8_t* valid, int64_t n, const void* w_in,
                  const void* w_out, int n_local, float residual_multiplier, void* h_out,
                  int64_t* topk_idx_out, void* topk_gate_out, void* stream);

/*
 * Post-attention RMSNorm of the MoE block: x = w * (h * rsqrt(mean(h^2) + eps)),
 * in the model dtype with the reference's rounding points.
 *   replaces: rms_norm (miniep/modeling.py:51-52) as called at :192
 * h, x: (n, H) rows starting on 16-byte boundaries; w: (H,).
 */
int mep_rmsnorm(mep_ctx* ctx, const void* h, const void* w, float eps, int64_t n, void* x_out,
                void* stream);

/*
 * The MoE half of Block.forward from the residual stream alone: x = rms_norm(h),
 * router, MoE layer step, h_out = h + moe(x) * residual_multiplier.
 *   replaces: Block.forward lines miniep/modeling.py:192-197
 * x_out: (n, H) device scratch the caller owns (receives the normalised rows);
 * topk_idx_out / topk_gate_out as for mep_moe_block.
 */
int mep_moe_block_from_h(mep_ctx* ctx, int layer, const void* h, const void* norm_w, float eps,
                         const void* router_w, const float* bias, const uint8_t* valid,
                         int64_t n, const void* w_in, const void* w_out, int n_local,
                         float residual_multiplier, void* h_out, void* x_out,
                         int64_t* topk_idx_out, void* topk_gate_out, void* stream);

/*
 * The layer step as separately launchable stages, in this order, for stage
 * timing and profiling (mep_moe_forward runs exactly these):
 *   mep_route       flatten_topk + route_counts + dest_ranks + counts publish
 *                   (modeling.py:107-117, ep.py:211-224)
 *   mep_dispatch    wait for counts, place rows at their owners, wait until
 *                   every rank's rows for this rank have landed (ep.py:224-226)
 *   mep_expert_ffn  grouped SwiGLU, output rows stored back at their sources
 *                   (ep.py:229-234, run_experts modeling.py:83-104)
 *   mep_combine     wait for results, gate * y summed in slot order, optional
 *                   residual (ep.py:237-242, modeling.py:120-128, :197);
 *                   h / h_out may be NULL, out may be NULL when h_out is set.
 */
int mep_route(mep_ctx* ctx, int layer, const int64_t* topk_idx, const uint8_t* valid, int64_t n,
              int n_local, void* stream);
int mep_dispatch(mep_ctx* ctx, const void* x, const int64_t* topk_idx, int64_t n, void* stream);
int mep_expert_ffn(mep_ctx* ctx, const void* w_in, const void* w_out, int n_local, void* stream);
int mep_combine(mep_ctx* ctx, const void* topk_gate, const uint8_t* valid, int64_t n,
                const void* h, float residual_multiplier, void* out, void* h_out, void* stream);

/*
 * Routing statistics (synchronises `stream`): route_counts_out (host, L x E
 * int64), recv_tokens_per_layer_out (host, L int64), either may be NULL.
 *   replaces: EPStats.route_counts / recv_tokens_per_layer / snapshot
 *             (miniep/ep.py:164-183, updates ep.py:216-217, 244-246)
 */
int mep_read_stats(mep_ctx* ctx, int64_t* route_counts_out, int64_t* recv_tokens_per_layer_out,
                   void* stream);
int mep_reset_stats(mep_ctx* ctx, void* stream);

/* Receive rows of the last layer step on this rank (synchronises). */
int mep_last_recv_rows(mep_ctx* ctx, int64_t* rows_out, void* stream);

/*
 * Device error word: MEP_OK, or MEP_ERR_DEVICE with the cause in
 * mep_last_error (and the word cleared). Call after synchronising.
 *   replaces: the reference's residency assert (miniep/ep.py:230) and gloo's
 *             collective timeouts
 */
int mep_check(mep_ctx* ctx);

/*
 * Options: "force_simt" (1 = CUDA-core expert GEMMs for bf16 too),
 * "timeout_ms" (bound on every cross-rank wait, default 10000),
 * "tc_single_cta" (1 = one CTA per 128-row expert tile instead of CTA pairs),
 * "timeline" (1 = kernels stamp the step timeline read by mep_read_timeline;
 * launches enqueued or captured while it is 0 stamp nothing),
 * "dispatch_per_warp" (1, default = one warp places each token; 0 = the
 * streaming dispatch engine), "router_no_tc" (1 = the warp router even for
 * batches the tcgen05 router covers), "ffn_ast" (1 = A-stationary GEMM2 for
 * CTA pairs), "ffn_prefetch" (1 = the expert GEMMs prefetch their next
 * tile's activation rows into L2). "ffn_ast" and "ffn_prefetch" default to
 * 0: both measured slower on the bench workload and stay for experiments.
 */
int mep_set_option(mep_ctx* ctx, const char* name, int64_t value);

/*
 * Step timeline (profiling aid, no counterpart in the reference): with the
 * "timeline" option set, each stage of a layer step records %globaltimer
 * stamps in nanoseconds: slot S = the stage's start (its first CTA), S + 1 =
 * its end (the last of its CTAs to finish); the single-point slots mark when
 * a wait ended. mep_read_timeline copies MEP_TL_SLOTS stamps to `out` (host),
 * synchronises `stream`, then zeroes the stamps. A stage that did not run
 * reads 0. Stamps of different GPUs come from different clocks; compare each
 * rank's stamps with its own MEP_TL_BARRIER_END.
 */
#define MEP_TL_BARRIER_END 0  /* mep_barrier: every rank arrived */
#define MEP_TL_NORM 1         /* k_rmsnorm start, end */
#define MEP_TL_ROUTER 3       /* router start, end */
#define MEP_TL_ROUTE 5        /* routing start, end */
#define MEP_TL_COUNTS_SENT 7  /* this rank's counts stored at every rank */
#define MEP_TL_LAYOUT 8       /* every rank's counts in, receive layout written */
#define MEP_TL_DISPATCH 9     /* dispatch start, end */
#define MEP_TL_DATA_IN 11     /* every rank's rows for this rank landed */
#define MEP_TL_FANOUT 12      /* landing-row fan-out start, end */
#define MEP_TL_GEMM1 14       /* expert GEMM1 + SwiGLU start, end */
#define MEP_TL_GEMM2 16       /* expert GEMM2 + return stores start, end */
#define MEP_TL_RESULTS_IN 18  /* every owner's results for this rank landed */
#define MEP_TL_COMBINE 19     /* combine start, end */
#define MEP_TL_ROUTE_HIST 21  /* routing: the last CTA's histogram written */
#define MEP_TL_ROUTE_SYNC 22  /* routing: the finalizing CTA left the grid barrier */
#define MEP_TL_SLOTS 24
int mep_read_timeline(mep_ctx* ctx, uint64_t* out, void* stream);

/*
 * Rank barrier on the device: this rank's kernel raises its flag on every
 * rank and waits (bounded by the context timeout) until every rank has done
 * the same, so the streams of all ranks leave it together without a host
 * round trip. No counterpart in the reference (its ranks meet in host
 * collectives); used to start timed steps on all GPUs at the same moment.
 * Every rank must call it the same number of times.
 */
int mep_barrier(mep_ctx* ctx, void* stream);

/*
 * Test hook for bounded waits: launches one wait on this rank's counts flag
 * for `target`; if nothing raises it within timeout_ms the kernel records a
 * device error and returns, so the context stays usable.
 */
int mep_debug_wait(mep_ctx* ctx, uint32_t target, int64_t timeout_ms, void* stream);

/*
 * mep_dest_ranks without a context and without any device allocation.
 * This entry point has no counterpart in the reference. It exists for callers
 * that cannot call cudaMalloc: a serving process that has handed all free HBM
 * to its own memory pool (a later cudaMalloc fails or fragments that pool),
 * or host code on a latency-critical path, where cudaMalloc/cudaFree would
 * synchronise the device. Results equal mep_dest_ranks for the same table,
 * round-robin state and ids.
 *   table (host, E x rmax int64) / n_rep (host, E int64): one layer's
 *     placement, as for mep_set_placement; world: ranks in the placement;
 *   rr (device, E int64): round-robin state of that layer, updated in place
 *     (zero it to reset, like Placement.reset_rr); any value is accepted, the
 *     replica being (rr + occurrence) mod n_rep taken non-negative, as
 *     Python's % gives it;
 *   expert_ids / dest_out (device, m int64), m <= 65536.
 * An id outside [0, E) gets destination -1 and does not advance the
 * round-robin state, as in mep_dest_ranks; but where mep_dest_ranks also
 * records a device error for mep_check, this entry point has no context to
 * record it in and reports nothing, so validate ids that can be out of range.
 * Its intermediate buffers live in one fixed array of about 650 KiB that
 * every GPU loading this library keeps until the process exits. All calls
 * share that array: calls whose kernels can overlap on one GPU race, so the
 * caller must serialise them. Every call copies the placement table from
 * host stack memory (pageable) with cudaMemcpyAsync, and the first call on
 * each device also looks up the array's device address, so no call may be
 * made while its stream is being captured. Larger calls fail with
 * MEP_ERR_INVALID; messages come from mep_last_error(NULL).
 */
int mep_dest_ranks_noalloc(int num_experts, int world, const int64_t* table,
                           const int64_t* n_rep, int rmax, int64_t* rr,
                           const int64_t* expert_ids, int64_t m, int64_t* dest_out,
                           void* stream);

#ifdef __cplusplus
}
#endif

#endif /* MINIEP_B200_H_ */
