// Dispatch and combine.
//
// Dispatch (ep.py:223-226): every kept entry's hidden row is stored straight
// into the destination rank's receive buffer at its final, expert-grouped
// position (peer stores over NVLink for remote ranks, local stores for this
// rank), together with a 4-byte tag (source rank, flat entry index) that
// tells the destination where the expert output must go back to. There is no
// send-side staging buffer and no separate permute pass.
//
// Combine (ep.py:234-242, scatter_combine modeling.py:120-128, residual
// modeling.py:197): the expert outputs arrive in this rank's (token, slot)
// landing buffer; each token sums gate * y over its slots in slot order
// 0..k-1 in fp32 (each product rounded to the model dtype first, as the
// reference multiplies in the model dtype), rounds once, and optionally adds
// the scaled residual. No atomics, so the result does not depend on the
// placement or on the number of ranks.
#include <cstdint>
#include "mep_device.cuh"

namespace mep {
namespace {

using bf16 = __nv_bfloat16;

// Signal "this kernel's stores are done" to every rank: flag slot
// [flag_base + rank] on each peer is raised to `seq` by the last CTA to finish.
// The CTAs count in kDoneGroups group counters (CTA b in group b % 32, each
// counter on its own cache line) and the last CTA of each group counts in
// done_ctr[0], so a grid of thousands of CTAs does not queue on one address.
__device__ __forceinline__ void grid_done_signal(unsigned int* done_ctr, const PeerPtrs& peers,
                                                 int world, int rank, int flag_base,
                                                 const uint32_t* seq) {
  if (world == 1) return;  // one rank: the next kernels follow in stream order
  __syncthreads();  // this CTA's stores happen before thread 0's fence below
  if (threadIdx.x == 0) {
    const unsigned grid = gridDim.x, g = blockIdx.x % kDoneGroups;
    const unsigned members = grid / kDoneGroups + (g < grid % kDoneGroups ? 1u : 0u);
    const unsigned groups = grid < kDoneGroups ? grid : kDoneGroups;
    unsigned int* grp = done_ctr + kDoneGroupBase + g * kDoneGroupStride;
    fence_acq_rel_sys();  // this CTA's stores (peers' rows included) before its count
    if (atomicAdd(grp, 1u) == members - 1) {
      *grp = 0u;               // the group is complete: reset for the next launch
      fence_acq_rel_gpu();  // the group's counts (this GPU) before the count below
      if (atomicAdd(done_ctr, 1u) == groups - 1) {
        fence_acq_rel_sys();
        const uint32_t step = *seq;
        for (int d = 0; d < world; ++d) st_relaxed_sys(peers.flags[d] + flag_base + rank, step);
        *done_ctr = 0u;
      }
    }
  }
}

// Entry f (a token's slot): its destination rank my_d and row my_pos in that
// rank's receive buffer (my_d = -1: not routed, or the destination would
// overflow, which the layout pass reported), its tag (source rank, entry)
// stored at the destination, and its row in this rank's return buffer,
// written back over ent_grp[f] (-1 when not routed) for the combine.
__device__ __forceinline__ void resolve_slot(int64_t f, int rank, const int64_t* topk_idx,
                                             const int32_t* ent_dest, int32_t* ent_grp,
                                             const Layout* lay, const PeerPtrs& peers, int& my_d,
                                             int64_t& my_pos) {
  const int d = ent_dest[f];
  int ret_row = -1;
  if (d >= 0) {
    const int e = (int)topk_idx[f];
    const int off = lay->dst_off[d * kMaxExperts + e];
    if (off >= 0) {
      const int grp = ent_grp[f];
      my_d = d;
      my_pos = (int64_t)off + grp;
      peers.recv_meta[d][my_pos] = (rank << 24) | (int32_t)f;
      ret_row = lay->ret_off[d * kMaxExperts + e] + grp;
    }
  }
  ent_grp[f] = ret_row;
}

// Dispatch, one warp per token: lanes s < k resolve slot s's destination row
// in the destination's expert-grouped layout and store the 4-byte tag there
// (source rank, flat entry index). The warp loads the token's row into one of
// its shared-memory row buffers and lane 0 issues bulk copies (cp.async.bulk,
// shared -> global, the TMA engine): one per slot that stays on this rank,
// straight into its receive row, and ONE per distinct remote destination rank
// into that rank's landing buffer [this rank][token], however many of the
// token's slots go there (the receiver fans it out locally). The copies run
// asynchronously; a row buffer is reused only once its earlier copies have
// read it.
constexpr int kDispatchWarps = 4;
constexpr int kDispatchBufs = 3;  // row buffers per warp


__global__ void __launch_bounds__(32 * kDispatchWarps) k_dispatch(
    int64_t n, int topk, int row_bytes, int world, int rank, int64_t max_tokens,
    const uint8_t* __restrict__ x, const int64_t* __restrict__ topk_idx,
    const int32_t* __restrict__ ent_dest, int32_t* __restrict__ ent_grp,
    const Layout* __restrict__ lay, PeerPtrs peers, unsigned int* done_ctr, const uint32_t* seq,
    uint64_t* tl) {
  extern __shared__ __align__(128) uint8_t dsmem[];
  const int lane = lane_id(), wp = warp_id();
  tl_begin(tl, kTlDispatch);
  uint8_t* bufs = dsmem + (size_t)wp * kDispatchBufs * row_bytes;
  const int64_t stride = (int64_t)gridDim.x * kDispatchWarps;
  const int vec = row_bytes >> 4;
  int buf = 0;
  for (int64_t t = (int64_t)blockIdx.x * kDispatchWarps + wp; t < n; t += stride) {
    int my_d = -1;
    int64_t my_pos = 0;
    if (lane < topk)
      resolve_slot(t * topk + lane, rank, topk_idx, ent_dest, ent_grp, lay, peers, my_d, my_pos);
    // local slots each need their own row; a remote rank needs the row once
    bool first_remote = my_d >= 0 && my_d != rank;
    for (int j = 0; j < topk; ++j) {
      const int dj = __shfl_sync(0xffffffffu, my_d, j);
      if (j < lane && dj == my_d) first_remote = false;
    }
    const unsigned remote = __ballot_sync(0xffffffffu, first_remote);
    const unsigned local = __ballot_sync(0xffffffffu, my_d == rank);
    if ((remote | local) == 0u) continue;
    uint8_t* row = bufs + (size_t)buf * row_bytes;
    // the buffer's previous copies (issued kDispatchBufs tokens ago) must have read it
    if (lane == 0)
      asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(kDispatchBufs - 1) : "memory");
    __syncwarp();
    const uint4* src = reinterpret_cast<const uint4*>(x + t * (int64_t)row_bytes);
    for (int c = lane; c < vec; c += 32) reinterpret_cast<uint4*>(row)[c] = __ldg(src + c);
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // smem writes -> bulk copies
    __syncwarp();
    for (int s = 0; s < topk; ++s) {
      const int d = __shfl_sync(0xffffffffu, my_d, s);
      const int64_t pos = __shfl_sync(0xffffffffu, my_pos, s);
      uint8_t* dst = nullptr;
      if ((local >> s) & 1u)
        dst = static_cast<uint8_t*>(peers.recv_x[rank]) + pos * row_bytes;
      else if ((remote >> s) & 1u)
        dst = static_cast<uint8_t*>(peers.land[d]) + ((int64_t)rank * max_tokens + t) * row_bytes;
      if (lane == 0 && dst)
        asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst),
                     "r"(smem_u32(row)), "r"(row_bytes)
                     : "memory");
    }
    if (lane == 0) asm volatile("cp.async.bulk.commit_group;" ::: "memory");
    buf = buf + 1 == kDispatchBufs ? 0 : buf + 1;
  }
  // every copy of this warp has completed (written) before the completion signal
  if (lane == 0) {
    asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
    asm volatile("fence.proxy.async.global;" ::: "memory");
  }
  grid_done_signal(done_ctr, peers, world, rank, world, seq);
  tl_end(tl, kTlDispatch + 1);
}

// Dispatch as a streaming engine, one CTA per SM over a contiguous token
// range. Warp 0 (one lane) bulk-loads the CTA's token rows, in order, into a
// ring of shared-memory slots (cp.async.bulk global -> shared, completing on
// the slot's `full` mbarrier). Warps 1.. take the tokens round-robin: lanes
// s < k resolve slot s's destination and store its tag (as k_dispatch does),
// then lane 0 waits for the row and issues its bulk copies shared -> global
// (each local slot's receive row, one landing row per distinct remote rank)
// as one bulk group. A placing warp keeps kDspPending groups in flight and
// releases a ring slot (its `empty` mbarrier) once that slot's copies have
// read shared memory, so the HBM reads, the local writes and the NVLink
// writes of many tokens overlap. Every wait is bounded.
// Progress: the loader can wait for a slot that a placing warp still holds
// only while the ring holds fewer than (placing warps) x (groups in flight
// - 1) slots, so the host sizes the groups in flight to the ring
// (dispatch_pending, at most kDspPending).
constexpr int kDspWarps = 8;      // warp 0 loads, warps 1..7 place
constexpr int kDspPending = 4;    // bulk groups a placing warp keeps in flight, at most
constexpr int kDspMaxSlots = 64;  // ring slots (fewer when the rows are long)
constexpr unsigned long long kDspWaitNs = 2000000000ull;
constexpr int kDspChunkTok = 256;  // tokens whose slots are resolved together

__device__ __forceinline__ void bulk_wait_read_pending(int keep) {
  switch (keep) {  // wait_group.read takes an immediate
    case 0: asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); break;
    case 1: asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory"); break;
    case 2: asm volatile("cp.async.bulk.wait_group.read 2;" ::: "memory"); break;
    default: asm volatile("cp.async.bulk.wait_group.read 3;" ::: "memory"); break;
  }
}

__global__ void __launch_bounds__(32 * kDspWarps, 1) k_dispatch_stream(
    int64_t n, int topk, int row_bytes, int world, int rank, int64_t max_tokens, int nslots,
    int pending, const uint8_t* __restrict__ x, const int64_t* __restrict__ topk_idx,
    const int32_t* __restrict__ ent_dest, int32_t* __restrict__ ent_grp,
    const Layout* __restrict__ lay, PeerPtrs peers, unsigned int* done_ctr, const uint32_t* seq,
    int* err, uint64_t* tl) {
  extern __shared__ __align__(128) uint8_t dsmem[];
  __shared__ uint64_t full[kDspMaxSlots], empty[kDspMaxSlots];
  __shared__ int pend_slot[kDspWarps][kDspPending];
  __shared__ int8_t s_dst[kDspChunkTok * kMaxTopk];   // a chunk's resolved slots
  __shared__ int32_t s_pos[kDspChunkTok * kMaxTopk];
  __shared__ int abort_flag;
  __shared__ int chunk_go;  // placing warps: go on to the next chunk
  const int lane = lane_id(), wp = warp_id();
  tl_begin(tl, kTlDispatch);
  const int64_t per = (n + gridDim.x - 1) / gridDim.x;
  const int64_t t0 = min((int64_t)blockIdx.x * per, n);
  const int64_t cnt = min(t0 + per, n) - t0;
  if (threadIdx.x == 0) {
    for (int sl = 0; sl < nslots; ++sl) {
      mbar_init(&full[sl], 1);
      mbar_init(&empty[sl], 1);
    }
    abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  if (wp == 0) {
    if (lane == 0) {
      int64_t issued = 0;
      for (int64_t i = 0; i < cnt; ++i) {
        const int sl = (int)(i % nslots);
        const uint32_t ph = (uint32_t)(i / nslots) & 1u;
        if (!mbar_wait_for(&empty[sl], ph ^ 1u, kDspWaitNs, &abort_flag)) {
          set_err(err, kErrPipeline);
          break;
        }
        mbar_expect_tx(&full[sl], (uint32_t)row_bytes);
        bulk_load_g2s(dsmem + (size_t)sl * row_bytes, x + (t0 + i) * (int64_t)row_bytes,
                      (uint32_t)row_bytes, &full[sl]);
        issued = i + 1;
      }
      // no load may still be writing shared memory when the CTA exits (after
      // an abort the placing warps did not wait for every row): wait, bounded,
      // for the last load issued into each slot
      for (int sl = 0; sl < nslots && sl < issued; ++sl) {
        const int64_t last = sl + (issued - 1 - sl) / nslots * nslots;
        mbar_wait_for(&full[sl], (uint32_t)(last / nslots) & 1u, kDspWaitNs, nullptr);
      }
    }
  } else {
    // placing warps: resolve a chunk's slots together (all of their global
    // loads in flight at once), then place its tokens round-robin
    const int ptid = threadIdx.x - 32, nplace = (kDspWarps - 1) * 32;
    int pend = 0, head = 0;  // lane 0: groups issued and not yet known read
    bool ok_all = true;
    for (int64_t c0 = 0; c0 < cnt && ok_all; c0 += kDspChunkTok) {
      const int ct = (int)min((int64_t)kDspChunkTok, cnt - c0);
      for (int i = ptid; i < ct * topk; i += nplace) {
        int d = -1;
        int64_t pos = 0;
        resolve_slot((t0 + c0) * topk + i, rank, topk_idx, ent_dest, ent_grp, lay, peers, d, pos);
        s_dst[i] = (int8_t)d;
        s_pos[i] = (int32_t)pos;
      }
      asm volatile("bar.sync 1, %0;" ::"n"((kDspWarps - 1) * 32) : "memory");
      for (int i = wp - 1; i < ct; i += kDspWarps - 1) {
        const int64_t ti = c0 + i;  // token index within this CTA's range
        const int64_t t = t0 + ti;
        const int sl = (int)(ti % nslots);
        const uint32_t ph = (uint32_t)(ti / nslots) & 1u;
        const int my_d = lane < topk ? s_dst[i * topk + lane] : -1;
        const int64_t my_pos = lane < topk ? s_pos[i * topk + lane] : 0;
        bool first_remote = my_d >= 0 && my_d != rank;
        for (int j = 0; j < topk; ++j) {
          const int dj = __shfl_sync(0xffffffffu, my_d, j);
          if (j < lane && dj == my_d) first_remote = false;
        }
        const unsigned remote = __ballot_sync(0xffffffffu, first_remote);
        const unsigned local = __ballot_sync(0xffffffffu, my_d == rank);
        int ok = 1;
        if (lane == 0) ok = mbar_wait_for(&full[sl], ph, kDspWaitNs, &abort_flag);
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (!ok) {
          if (lane == 0) set_err(err, kErrPipeline);
          ok_all = false;
          break;
        }
        const uint8_t* row = dsmem + (size_t)sl * row_bytes;
        for (int s = 0; s < topk; ++s) {
          const int d = __shfl_sync(0xffffffffu, my_d, s);
          const int64_t pos = __shfl_sync(0xffffffffu, my_pos, s);
          if (lane == 0) {
            if ((local >> s) & 1u)
              bulk_store_s2g(static_cast<uint8_t*>(peers.recv_x[rank]) + pos * row_bytes, row,
                             (uint32_t)row_bytes);
            else if ((remote >> s) & 1u)
              bulk_store_s2g(static_cast<uint8_t*>(peers.land[d]) +
                                 ((int64_t)rank * max_tokens + t) * row_bytes,
                             row, (uint32_t)row_bytes);
          }
        }
        if (lane == 0) {
          asm volatile("cp.async.bulk.commit_group;" ::: "memory");  // may be empty
          pend_slot[wp][(head + pend) % kDspPending] = sl;
          if (++pend > pending - 1) {
            // all but the newest pending-1 groups have read shared memory
            bulk_wait_read_pending(pending - 1);
            mbar_arrive(&empty[pend_slot[wp][head]]);
            head = (head + 1) % kDspPending;
            --pend;
          }
        }
        __syncwarp();
      }
      // every placing warp is done with this chunk's slots (also after an
      // abort: every placing warp reaches both barriers of a chunk); one
      // thread reads the abort flag so that all take the same branch
      asm volatile("bar.sync 1, %0;" ::"n"((kDspWarps - 1) * 32) : "memory");
      if (ptid == 0) chunk_go = !*(volatile int*)&abort_flag;
      asm volatile("bar.sync 1, %0;" ::"n"((kDspWarps - 1) * 32) : "memory");
      ok_all = chunk_go != 0;
    }
    if (lane == 0) {
      asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");  // every copy written
      asm volatile("fence.proxy.async.global;" ::: "memory");
    }
  }
  grid_done_signal(done_ctr, peers, world, rank, world, seq);
  tl_end(tl, kTlDispatch + 1);
}

// Fan-out on the receiver: once every rank's dispatch has signalled its rows
// for this rank (data flags [W, 2W), bounded wait), every receive row whose
// tag names another rank is copied from that rank's landing row
// [src][token] (one warp per row).
__global__ void __launch_bounds__(256) k_fanout(int row_bytes, int topk, int rank, int world,
                                                int64_t max_tokens, const Layout* __restrict__ lay,
                                                const int32_t* __restrict__ meta,
                                                const uint8_t* __restrict__ land,
                                                uint8_t* __restrict__ recv_x,
                                                const uint32_t* flags, const uint32_t* seq,
                                                WaitCfg wc, uint64_t* tl) {
  __shared__ int s_prefix[kMaxExperts + 1], s_base[kMaxExperts], s_rows[kMaxExperts];
  __shared__ int arrived;
  tl_begin(tl, kTlFanout);
  if (threadIdx.x == 0) arrived = 1;
  __syncthreads();
  if (threadIdx.x < world && !wait_flag(flags + world + threadIdx.x, *seq, kErrWaitData, wc))
    arrived = 0;
  __syncthreads();
  if (!arrived) return;  // the error word is set; the step fails as a whole
  if (blockIdx.x == 0 && threadIdx.x == 0) tl_mark(tl, kTlDataIn);
  const int nl = lay->n_local;
  for (int i = threadIdx.x; i <= nl; i += blockDim.x) s_prefix[i] = lay->tile_prefix[i];
  for (int i = threadIdx.x; i < nl; i += blockDim.x) {
    s_base[i] = lay->seg_base[i];
    s_rows[i] = lay->seg_rows[i];
  }
  __syncthreads();
  const int64_t total = (int64_t)lay->total_mtiles * kRowAlign;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  const int lane = lane_id(), vec = row_bytes >> 4;
  for (int64_t w = (int64_t)blockIdx.x * (blockDim.x >> 5) + warp_id(); w < total; w += warps) {
    const int tile = (int)(w / kRowAlign);
    int j = 0;
    while (j + 1 < nl && s_prefix[j + 1] <= tile) ++j;
    const int local = (tile - s_prefix[j]) * kRowAlign + (int)(w % kRowAlign);
    if (local >= s_rows[j]) continue;
    const int64_t p = (int64_t)s_base[j] + local;
    const int32_t mt = meta[p];
    const int src = mt >> 24;
    if (src == rank) continue;
    const int64_t t = (mt & 0xffffff) / topk;
    const uint4* from = reinterpret_cast<const uint4*>(land + ((int64_t)src * max_tokens + t) * row_bytes);
    uint4* to = reinterpret_cast<uint4*>(recv_x + p * row_bytes);
    for (int c = lane; c < vec; c += 32) to[c] = from[c];
  }
  tl_end(tl, kTlFanout + 1);
}

// Rank barrier: raise barrier flag [3W + rank] on every rank to the next
// barrier number, then wait for all W flags of this rank to reach it.
__global__ void k_rank_barrier(PeerPtrs peers, int world, int rank, uint32_t* bar_seq,
                               const uint32_t* flags, WaitCfg wc, uint64_t* tl) {
  const uint32_t s = *bar_seq + 1u;
  if (threadIdx.x < world) st_release_sys(peers.flags[threadIdx.x] + 3 * world + rank, s);
  if (threadIdx.x < world) wait_flag(flags + 3 * world + threadIdx.x, s, kErrWaitBarrier, wc);
  __syncthreads();
  if (threadIdx.x == 0) {
    *bar_seq = s;
    tl_mark(tl, kTlBarrierEnd);
  }
}

__global__ void k_wait_flags(const uint32_t* flags, int first, int world, const uint32_t* seq,
                             uint32_t target, int code, WaitCfg wc, uint64_t* tl, int tl_slot) {
  const uint32_t step = seq ? *seq : target;
  if (threadIdx.x < world) wait_flag(flags + first + threadIdx.x, step, code, wc);
  if (tl) {
    __syncthreads();
    if (threadIdx.x == 0) tl_mark(tl, tl_slot);
  }
}

template <typename T>
struct Vec16 {
  static constexpr int N = 16 / sizeof(T);
};

template <typename T>
__device__ __forceinline__ void unpack16(const uint4& v, float (&o)[Vec16<T>::N]);
template <>
__device__ __forceinline__ void unpack16<float>(const uint4& v, float (&o)[4]) {
  o[0] = __uint_as_float(v.x);
  o[1] = __uint_as_float(v.y);
  o[2] = __uint_as_float(v.z);
  o[3] = __uint_as_float(v.w);
}
template <>
__device__ __forceinline__ void unpack16<bf16>(const uint4& v, float (&o)[8]) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    o[2 * i] = __uint_as_float(w[i] << 16);
    o[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
  }
}
template <typename T>
__device__ __forceinline__ uint4 pack16(const float (&o)[Vec16<T>::N]);
template <>
__device__ __forceinline__ uint4 pack16<float>(const float (&o)[4]) {
  return make_uint4(__float_as_uint(o[0]), __float_as_uint(o[1]), __float_as_uint(o[2]),
                    __float_as_uint(o[3]));
}
template <>
__device__ __forceinline__ uint4 pack16<bf16>(const float (&o)[8]) {
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const __nv_bfloat162 p = __floats2bfloat162_rn(o[2 * i], o[2 * i + 1]);
    w[i] = *reinterpret_cast<const uint32_t*>(&p);
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}

// acc += model_dtype(y * g), element-wise over one 16-byte vector. For bf16
// the products are taken two at a time with bf16x2 multiplies, which round
// the exact product to bf16 exactly as multiplying in fp32 and rounding does
// (a product of two bf16 values is exact in fp32).
template <typename T>
__device__ __forceinline__ void add_gated(float (&acc)[Vec16<T>::N], const uint4& raw, float g);
template <>
__device__ __forceinline__ void add_gated<float>(float (&acc)[4], const uint4& raw, float g) {
  acc[0] += __uint_as_float(raw.x) * g;
  acc[1] += __uint_as_float(raw.y) * g;
  acc[2] += __uint_as_float(raw.z) * g;
  acc[3] += __uint_as_float(raw.w) * g;
}
template <>
__device__ __forceinline__ void add_gated<bf16>(float (&acc)[8], const uint4& raw, float g) {
  const __nv_bfloat162 g2 = __float2bfloat162_rn(g);  // g is a bf16 value: exact
  const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const __nv_bfloat162 p = __hmul2(*reinterpret_cast<const __nv_bfloat162*>(&w[i]), g2);
    const float2 f = __bfloat1622float2(p);
    acc[2 * i] += f.x;
    acc[2 * i + 1] += f.y;
  }
}

template <typename T, int KMAX>
__device__ __forceinline__ void combine_body(int64_t n, int topk, int H, int world,
                                             const T* __restrict__ ret,
                                             const int32_t* __restrict__ ent_ret,
                                             const T* __restrict__ gate,
                                             const uint8_t* __restrict__ valid,
                                             const T* __restrict__ h, float rm,
                                             T* __restrict__ out, T* __restrict__ h_out,
                                             const uint32_t* flags, const uint32_t* seq,
                                             WaitCfg wc, uint64_t* tl) {
  constexpr int V = Vec16<T>::N;
  tl_begin(tl, kTlCombine);
  // expert outputs from every rank (one rank: GEMM2 precedes in stream order)
  if (world > 1 && threadIdx.x < world)
    wait_flag(flags + 2 * world + threadIdx.x, *seq, kErrWaitDone, wc);
  __syncthreads();
  tl_begin(tl, kTlResultsIn);
  const int lane = lane_id();
  const int64_t warps_total = (int64_t)gridDim.x * (blockDim.x >> 5);
  const int nvec = H / V;
  for (int64_t t = (int64_t)blockIdx.x * (blockDim.x >> 5) + warp_id(); t < n; t += warps_total) {
    const bool keep = valid == nullptr || valid[t] != 0;
    // return row of each slot (-1: the entry was not routed)
    const int my_row = (keep && lane < topk) ? ent_ret[t * topk + lane] : -1;
    float g[KMAX];
    int row[KMAX];
#pragma unroll
    for (int s = 0; s < KMAX; ++s) {
      row[s] = __shfl_sync(0xffffffffu, my_row, s < topk ? s : 0);
      g[s] = (keep && s < topk && row[s] >= 0) ? Elt<T>::to_f(gate[t * topk + s]) : 0.f;
    }
    const uint4* rows = reinterpret_cast<const uint4*>(ret);
    for (int c = lane; c < nvec; c += 32) {
      float acc[V];
#pragma unroll
      for (int i = 0; i < V; ++i) acc[i] = 0.f;
      // the residual row and all of the token's slot rows in flight at once,
      // then the slots summed in slot order
      uint4 hr = make_uint4(0, 0, 0, 0);
      if (h_out) hr = reinterpret_cast<const uint4*>(h + t * (int64_t)H)[c];
      if (keep) {
        uint4 raw[KMAX];
#pragma unroll
        for (int s = 0; s < KMAX; ++s)
          raw[s] = (s < topk && row[s] >= 0) ? rows[(int64_t)row[s] * nvec + c]
                                             : make_uint4(0, 0, 0, 0);
#pragma unroll
        for (int s = 0; s < KMAX; ++s) {
          if (s < topk) add_gated<T>(acc, raw[s], g[s]);
        }
      }
      float o[V];
#pragma unroll
      for (int i = 0; i < V; ++i) o[i] = Elt<T>::round(acc[i]);
      if (out) reinterpret_cast<uint4*>(out + t * (int64_t)H)[c] = pack16<T>(o);
      if (h_out) {
        float hv[V];
        unpack16<T>(hr, hv);
        float r[V];
#pragma unroll
        for (int i = 0; i < V; ++i) r[i] = hv[i] + Elt<T>::round(o[i] * rm);
        reinterpret_cast<uint4*>(h_out + t * (int64_t)H)[c] = pack16<T>(r);
      }
    }
  }
  tl_end(tl, kTlCombine + 1);
}

// top-k <= 8: three CTAs per SM (more slot rows in flight per SM: measured
// 69.6 -> 65.5 us for 16384 tokens of shape (a), same results); top-16: the
// compiler's own register choice, its slot array needs them
template <typename T>
__global__ void __launch_bounds__(256, 3) k_combine8(int64_t n, int topk, int H, int world,
                                                     const T* __restrict__ ret,
                                                     const int32_t* __restrict__ ent_ret,
                                                     const T* __restrict__ gate,
                                                     const uint8_t* __restrict__ valid,
                                                     const T* __restrict__ h, float rm,
                                                     T* __restrict__ out, T* __restrict__ h_out,
                                                     const uint32_t* flags, const uint32_t* seq,
                                                     WaitCfg wc, uint64_t* tl) {
  combine_body<T, 8>(n, topk, H, world, ret, ent_ret, gate, valid, h, rm, out, h_out, flags, seq,
                     wc, tl);
}
template <typename T>
__global__ void __launch_bounds__(256) k_combine16(int64_t n, int topk, int H, int world,
                                                   const T* __restrict__ ret,
                                                   const int32_t* __restrict__ ent_ret,
                                                   const T* __restrict__ gate,
                                                   const uint8_t* __restrict__ valid,
                                                   const T* __restrict__ h, float rm,
                                                   T* __restrict__ out, T* __restrict__ h_out,
                                                   const uint32_t* flags, const uint32_t* seq,
                                                   WaitCfg wc, uint64_t* tl) {
  combine_body<T, kMaxTopk>(n, topk, H, world, ret, ent_ret, gate, valid, h, rm, out, h_out,
                            flags, seq, wc, tl);
}

}  // namespace

void launch_dispatch(int dtype, int64_t n, int topk, int hidden, int world, int rank,
                     int64_t max_tokens, const void* x, const int64_t* topk_idx,
                     const int32_t* ent_dest, int32_t* ent_grp, const Layout* layout,
                     const PeerPtrs& peers, unsigned int* done_ctr, const uint32_t* seq,
                     int num_sms, int per_warp, int* err, uint64_t* tl, cudaStream_t st) {
  const int row_bytes = hidden * (dtype == kBF16 ? 2 : 4);
  if (!per_warp) {
    // ring slots within ~180 KB of dynamic shared memory (the chunk's
    // resolved slots take another 20 KB of static shared memory)
    int nslots = (180 * 1024) / row_bytes;
    if (nslots > kDspMaxSlots) nslots = kDspMaxSlots;
    if (nslots < 2) nslots = 2;
    const size_t smem = (size_t)nslots * row_bytes;
    static size_t stream_smem_set = 0;
    if (smem > 48 * 1024 && smem > stream_smem_set) {
      cudaFuncSetAttribute(k_dispatch_stream, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)smem);
      stream_smem_set = smem;
    }
    // groups in flight per placing warp: the ring must hold more than
    // (placing warps) x (pending - 1) slots (see kDspWarps)
    int pending = (nslots - 1) / (kDspWarps - 1) + 1;
    if (pending > kDspPending) pending = kDspPending;
    k_dispatch_stream<<<(unsigned)num_sms, 32 * kDspWarps, smem, st>>>(
        n, topk, row_bytes, world, rank, max_tokens, nslots, pending,
        static_cast<const uint8_t*>(x),
        topk_idx, ent_dest, ent_grp, layout, peers, done_ctr, seq, err, tl);
    return;
  }
  const size_t smem = (size_t)kDispatchWarps * kDispatchBufs * row_bytes;
  static size_t smem_set = 0;
  if (smem > 48 * 1024 && smem > smem_set) {
    cudaFuncSetAttribute(k_dispatch, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    smem_set = smem;
  }
  // one warp per token up to the grid cap
  int64_t blocks = (n + kDispatchWarps - 1) / kDispatchWarps;
  if (blocks > (int64_t)num_sms * 16) blocks = (int64_t)num_sms * 16;
  if (blocks < 1) blocks = 1;
  k_dispatch<<<(unsigned)blocks, 32 * kDispatchWarps, smem, st>>>(
      n, topk, row_bytes, world, rank, max_tokens, static_cast<const uint8_t*>(x), topk_idx,
      ent_dest, ent_grp, layout, peers, done_ctr, seq, tl);
}

void launch_fanout(int dtype, int hidden, int topk, int rank, int world, int64_t max_tokens,
                   const Layout* layout, const int32_t* recv_meta, const void* land, void* recv_x,
                   const uint32_t* flags_local, const uint32_t* seq, WaitCfg wc, int num_sms,
                   uint64_t* tl, cudaStream_t st) {
  k_fanout<<<(unsigned)num_sms * 8, 256, 0, st>>>(hidden * (dtype == kBF16 ? 2 : 4), topk, rank,
                                                  world, max_tokens, layout, recv_meta,
                                                  static_cast<const uint8_t*>(land),
                                                  static_cast<uint8_t*>(recv_x), flags_local, seq,
                                                  wc, tl);
}

void launch_rank_barrier(const PeerPtrs& peers, int world, int rank, uint32_t* bar_seq,
                         const uint32_t* flags_local, WaitCfg wc, uint64_t* tl, cudaStream_t st) {
  k_rank_barrier<<<1, 32, 0, st>>>(peers, world, rank, bar_seq, flags_local, wc, tl);
}

void launch_wait_flags(const uint32_t* flags_local, int first, int world, const uint32_t* seq,
                       uint32_t target, int errcode, WaitCfg wc, uint64_t* tl, int tl_slot,
                       cudaStream_t st) {
  k_wait_flags<<<1, 32, 0, st>>>(flags_local, first, world, seq, target, errcode, wc, tl, tl_slot);
}

void launch_combine(int dtype, int64_t n, int topk, int hidden, int world, const void* ret_local,
                    const int32_t* ent_ret, const void* topk_gate, const uint8_t* valid, const void* h,
                    float residual_multiplier, void* out, void* h_out, const uint32_t* flags_local,
                    const uint32_t* seq, WaitCfg wc, int num_sms, uint64_t* tl, cudaStream_t st) {
  int64_t blocks = (n + 7) / 8;
  if (blocks > (int64_t)num_sms * 8) blocks = (int64_t)num_sms * 8;
  if (blocks < 1) blocks = 1;
  // slot rows in flight per lane: sized to top-k (8 or 16) to keep registers low
#define MEP_COMBINE(T, KM)                                                                  \
  k_combine##KM<T><<<(unsigned)blocks, 256, 0, st>>>(                                       \
      n, topk, hidden, world, static_cast<const T*>(ret_local), ent_ret,                       \
      static_cast<const T*>(topk_gate),                                                       \
      valid, static_cast<const T*>(h), residual_multiplier, static_cast<T*>(out),             \
      static_cast<T*>(h_out), flags_local, seq, wc, tl)
  static_assert(kMaxTopk == 16, "combine kernels are instantiated for top-8 and top-16");
  if (dtype == kBF16) {
    if (topk <= 8)
      MEP_COMBINE(bf16, 8);
    else
      MEP_COMBINE(bf16, 16);
  } else {
    if (topk <= 8)
      MEP_COMBINE(float, 8);
    else
      MEP_COMBINE(float, 16);
  }
#undef MEP_COMBINE
}

}  // namespace mep
