// Internal declarations shared by the CUDA translation units of libminiep_b200.
// Nothing here is part of the C ABI (include/miniep_b200.h is).
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>

#include "miniep_b200.h"

namespace mep {

constexpr int kMaxWorld = 8;      // ranks of one NVLink/NVSwitch box
constexpr int kMaxExperts = 128;  // experts per layer
constexpr int kMaxTopk = 16;
constexpr int kRowAlign = 128;    // expert segments in the receive buffer start on 128-row boundaries
constexpr int kRouteChunkTokens = 256;  // tokens per CTA in the routing scan
// completion counters of a context: [0] dispatch, [1] expert FFN, [2..3]
// routing grid barrier; from kDoneGroupBase, kDoneGroups dispatch group
// counters, one per 128-byte line (kDoneGroupStride words apart)
constexpr int kDoneGroups = 32;
constexpr int kDoneGroupBase = 32;
constexpr int kDoneGroupStride = 32;
constexpr int kDoneCounters = kDoneGroupBase + kDoneGroups * kDoneGroupStride;

enum DType : int { kF32 = 0, kBF16 = 1 };

// Step-timeline slots (the MEP_TL_* values of the public header).
enum TlSlot : int {
  kTlBarrierEnd = MEP_TL_BARRIER_END,
  kTlNorm = MEP_TL_NORM,
  kTlRouter = MEP_TL_ROUTER,
  kTlRoute = MEP_TL_ROUTE,
  kTlCountsSent = MEP_TL_COUNTS_SENT,
  kTlLayout = MEP_TL_LAYOUT,
  kTlDispatch = MEP_TL_DISPATCH,
  kTlDataIn = MEP_TL_DATA_IN,
  kTlFanout = MEP_TL_FANOUT,
  kTlGemm1 = MEP_TL_GEMM1,
  kTlGemm2 = MEP_TL_GEMM2,
  kTlResultsIn = MEP_TL_RESULTS_IN,
  kTlCombine = MEP_TL_COMBINE,
  kTlRouteHist = MEP_TL_ROUTE_HIST,
  kTlRouteSync = MEP_TL_ROUTE_SYNC,
  kTlSlots = MEP_TL_SLOTS,
};

// Device-side error word values (written to host-mapped memory).
enum DevErr : int {
  kErrNone = 0,
  kErrWaitCounts = 1,     // timed out waiting for a peer's routing counts
  kErrWaitData = 2,       // timed out waiting for a peer's dispatched rows
  kErrWaitDone = 3,       // timed out waiting for a peer's expert outputs
  kErrExpertId = 4,       // routing index outside [0, E)
  kErrCapacity = 5,       // a receive buffer would overflow
  kErrNotResident = 6,    // entry routed to a rank that does not hold the expert
  kErrWaitDebug = 7,      // the debug wait entry point timed out
  kErrPipeline = 8,       // a tensor-core pipeline barrier timed out
  kErrWaitBarrier = 9,    // timed out waiting for a peer at a rank barrier
};

// Receive-side layout and send offsets for one layer step, computed on the
// device after the routing counts of every rank are known.
struct Layout {
  int n_local;                       // experts resident on this rank
  int total_rows;                    // padded rows of the receive buffer in use
  int total_mtiles;                  // 128-row tiles over all local segments
  int recv_rows;                     // real (unpadded) rows received
  int seg_base[kMaxExperts];         // first padded row of local expert j
  int seg_rows[kMaxExperts];         // rows of local expert j
  int tile_prefix[kMaxExperts + 1];  // first 128-row tile of local expert j
  int local_expert[kMaxExperts];     // global id of local expert j
  int dst_off[kMaxWorld * kMaxExperts];  // [d][e]: first row this rank writes at rank d for expert e
  // Return buffer. Every rank receives its entries' expert outputs in (owner
  // rank d, expert e, index within the (d, e) group) order:
  int ret_off[kMaxWorld * kMaxExperts];  // [d][e]: first return row of the (d, e) group here
  // owner side, per local segment j: rows from source s start at row
  // src_begin[j][s] of the segment (src_begin[j][world] = the segment's
  // rows) and go to row ret_row[j][s] of source s's return buffer
  int src_begin[kMaxExperts * (kMaxWorld + 1)];
  int ret_row[kMaxExperts * kMaxWorld];
};

// Pointers every rank can reach (own and peers' symmetric buffers).
struct PeerPtrs {
  void* recv_x[kMaxWorld];     // expert-grouped receive rows
  void* land[kMaxWorld];       // token landing buffers: [src rank][max_tokens][H]
  int32_t* recv_meta[kMaxWorld];
  void* ret[kMaxWorld];        // return buffers: expert outputs in (owner, expert, group) order
  int32_t* cnt_in[kMaxWorld];
  uint32_t* flags[kMaxWorld];  // [0,W) counts, [W,2W) data, [2W,3W) done, [3W,4W) barrier
};

struct WaitCfg {
  int* err;                 // host-mapped error word
  unsigned long long timeout_ns;
};

// ---------------------------------------------------------------- router
// `tl` (every launcher below that takes it): the step timeline, or null when
// the context's timeline option is off (mep_device.cuh, tl_begin / tl_end)
// use_tc: allow the tcgen05 router from kRouterTcMinTokens tokens
constexpr int64_t kRouterTcMinTokens = 256;
void launch_router(int dtype, const void* x, const void* router_w, const float* bias,
                   int64_t n, int hidden, int experts, int topk, int64_t* idx_out,
                   void* gate_out, float* logits_out, int num_sms, int use_tc, int* err,
                   uint64_t* tl, cudaStream_t st);
// the tcgen05 router (mep_router_tc.cu): 0 when it ran, nonzero when the
// shape is not covered (bf16, E of 32 or 64, H a multiple of 64, 16-byte rows)
int launch_router_tc(int64_t n, int hidden, int experts, int topk, const void* x,
                     const void* router_w, const float* bias, int64_t* idx_out, void* gate_out,
                     float* logits_out, int num_sms, int* err, uint64_t* tl, cudaStream_t st);

// ---------------------------------------------------------------- RMSNorm
void launch_rmsnorm(int dtype, int64_t n, int hidden, const void* h, const void* w, float eps,
                    void* x, uint64_t* tl, cudaStream_t st);

// ---------------------------------------------------------------- routing
void launch_route(int64_t n, int topk, int experts, int world, int rank,
                  const int64_t* topk_idx, const uint8_t* valid,
                  const int32_t* owners_l, const int32_t* nrep_l, int64_t* rr_l,
                  int64_t* route_counts_l, int32_t* chunk_hist, int32_t* ent_dest,
                  int32_t* ent_grp, int32_t* my_counts, const PeerPtrs& peers,
                  uint32_t* seq, unsigned int* sync, int num_sms,
                  const int32_t* cnt_in_local, const uint32_t* flags_local,
                  int64_t* recv_per_layer_l, int64_t cap_rows, Layout* layout, WaitCfg wc,
                  uint64_t* tl, cudaStream_t st);

void launch_dest_only(int64_t m, int experts, const int64_t* expert_ids,
                      const int32_t* owners_l, const int32_t* nrep_l, int64_t* rr_l,
                      int32_t* chunk_hist, int32_t* ent_dest, int32_t* ent_grp,
                      int64_t* dest_out, WaitCfg wc, cudaStream_t st);


// ---------------------------------------------------------------- movement
void launch_dispatch(int dtype, int64_t n, int topk, int hidden, int world, int rank,
                     int64_t max_tokens,
                     const void* x, const int64_t* topk_idx, const int32_t* ent_dest,
                     int32_t* ent_grp, const Layout* layout, const PeerPtrs& peers,
                     unsigned int* done_ctr, const uint32_t* seq, int num_sms, int per_warp,
                     int* err, uint64_t* tl, cudaStream_t st);

// every rank raises its barrier flag on every peer, then waits (bounded) for all
void launch_rank_barrier(const PeerPtrs& peers, int world, int rank, uint32_t* bar_seq,
                         const uint32_t* flags_local, WaitCfg wc, uint64_t* tl, cudaStream_t st);

// waits for flags [first, first + world) to reach *seq (or `target` when seq is null)
// Receive rows that came from other ranks: once every rank's data flag for
// this step is up (bounded wait, timeline mark MEP_TL_DATA_IN), copy each
// from the landing buffer (row [src][token]) to its expert-segment row.
void launch_fanout(int dtype, int hidden, int topk, int rank, int world, int64_t max_tokens,
                   const Layout* layout, const int32_t* recv_meta, const void* land,
                   void* recv_x, const uint32_t* flags_local, const uint32_t* seq, WaitCfg wc,
                   int num_sms, uint64_t* tl, cudaStream_t st);

// `tl_slot`: timeline slot stamped when the wait ends (ignored when tl is null)
void launch_wait_flags(const uint32_t* flags_local, int first, int world, const uint32_t* seq,
                       uint32_t target, int errcode, WaitCfg wc, uint64_t* tl, int tl_slot,
                       cudaStream_t st);

void launch_combine(int dtype, int64_t n, int topk, int hidden, int world,
                    const void* ret_local, const int32_t* ent_ret, const void* topk_gate,
                    const uint8_t* valid,
                    const void* h, float residual_multiplier, void* out, void* h_out,
                    const uint32_t* flags_local, const uint32_t* seq, WaitCfg wc, int num_sms,
                    uint64_t* tl, cudaStream_t st);

// ---------------------------------------------------------------- expert FFN
struct FfnArgs {
  int dtype;
  int hidden, inter, world, rank;
  int64_t cap_rows;
  const void* recv_x;       // (cap_rows, H)  local receive buffer
  int64_t ret_rows;         // rows of every rank's return buffer (max_tokens * topk)
  void* act;                // (cap_rows, I)  SwiGLU activations
  const void* w_in;         // (E_l, 2I, H)
  const void* w_out;        // (E_l, H, I)
  const Layout* layout;
  PeerPtrs peers;
  unsigned int* done_ctr;
  const uint32_t* seq;      // device: sequence number of the current layer step
  int num_sms;
  int force_simt;           // 1: run the CUDA-core kernels even for bf16
  int tc_single_cta;        // 1: one CTA per 128x256 tile instead of CTA pairs per 256x256
  int ast;                  // 1: GEMM2 keeps a row tile's A resident across its N blocks
  int prefetch;             // 1: the GEMMs prefetch their next tile's A rows into L2
  int n_local_weights;      // leading extent of w_in / w_out
  int* err;                 // host-mapped device error word
  uint64_t* tl;             // step timeline or null
};
// Returns 0 on success, else a cudaError_t value or a negative code.
int launch_ffn(const FfnArgs& a, cudaStream_t st);
bool tc_shape_ok(int hidden, int inter);
int tc_init();  // resolves cuTensorMapEncodeTiled; 0 ok
// bf16 2D tensor map with 128-byte swizzle (mep_ffn.cu); 0 ok
int encode_bf16_2d(CUtensorMap* m, const void* base, uint64_t inner, uint64_t outer,
                   uint32_t box_inner, uint32_t box_outer);

}  // namespace mep
