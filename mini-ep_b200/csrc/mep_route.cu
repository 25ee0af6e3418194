// Routing of entries to ranks, without a host round trip:
//   * per-expert histogram of the kept entries            (ep.py:216-217, route_counts)
//   * stable occurrence index of every entry within its expert, in flat
//     (token-major, slot-minor) order over kept entries   (ep.py:86-93)
//   * destination rank by replica round-robin,
//     replica = (rr[e] + occurrence) % n_rep[e], then rr[e] += count[e]   (ep.py:76-96)
//   * per-(destination, expert) counts published to every rank, which is the
//     counts exchange of the reference (ep.py:120-124) done as peer stores
//   * the receive layout (expert segments in sorted local-expert order, each
//     source's rows in rank order inside a segment) computed identically on
//     every rank from the exchanged counts.
// flatten_topk's masking (modeling.py:107-117) is folded in: entries of
// invalid tokens are not counted, not routed, not sent.
//
// Index within a (destination, expert) group: the entries of expert e with
// occurrence w go to replica slot (rr0 + w) % n; the earlier entries with the
// same slot are w - n, w - 2n, ... >= 0, so the group index is w / n.
#include <cstdint>
#include "mep_device.cuh"

namespace mep {
namespace {

constexpr int kRouteThreads = kRouteChunkTokens;  // one token per thread in the histogram pass
constexpr int kRouteWarps = kRouteThreads / 32;
constexpr int kRoutePrefetch = 8;  // independent loads a thread keeps in flight

// the token of entry f: a 64-bit division, kept out of line so that the
// unrolled scans that never need it (no valid mask) stay short
__device__ __noinline__ int64_t entry_token(int64_t f, int k) { return f / k; }

__device__ __forceinline__ int entry_expert(const int64_t* idx, const uint8_t* valid, int64_t f,
                                            int k, int64_t n, int E, int* err) {
  if (f >= n * k) return -1;
  if (valid && !valid[entry_token(f, k)]) return -1;
  const int64_t e = idx[f];
  if (e < 0 || e >= E) {
    set_err(err, kErrExpertId);
    return -1;
  }
  return (int)e;
}

__global__ void __launch_bounds__(kRouteThreads) k_route_hist(int64_t n, int k, int E,
                                                              const int64_t* __restrict__ idx,
                                                              const uint8_t* __restrict__ valid,
                                                              int32_t* __restrict__ chunk_hist,
                                                              int* err) {
  __shared__ int h[kMaxExperts];
  for (int e = threadIdx.x; e < E; e += blockDim.x) h[e] = 0;
  __syncthreads();
  const int64_t t = (int64_t)blockIdx.x * kRouteChunkTokens + threadIdx.x;
  if (t < n) {
    for (int s = 0; s < k; ++s) {
      const int e = entry_expert(idx, valid, t * k + s, k, n, E, err);
      if (e >= 0) atomicAdd(&h[e], 1);
    }
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) chunk_hist[(int64_t)blockIdx.x * E + e] = h[e];
}

// Occurrence index (stable, flat order) -> destination rank and index within
// the (destination, expert) group. Entries of one chunk are walked by warps in
// rounds of 32 consecutive flat entries; lanes holding the same expert are
// ranked with __match_any_sync.
__global__ void __launch_bounds__(kRouteThreads) k_route_rank(
    int64_t n, int k, int E, const int64_t* __restrict__ idx, const uint8_t* __restrict__ valid,
    const int32_t* __restrict__ owners, const int32_t* __restrict__ nrep,
    const int64_t* __restrict__ rr, const int32_t* __restrict__ chunk_hist,
    int32_t* __restrict__ ent_dest, int32_t* __restrict__ ent_grp) {
  __shared__ int base[kMaxExperts];
  __shared__ int wcnt[kRouteWarps][kMaxExperts];
  __shared__ int wbase[kRouteWarps][kMaxExperts];
  __shared__ int rr_mod[kMaxExperts];
  const int wp = warp_id(), lane = lane_id();
  const int chunk = blockIdx.x;
  // prefix of the earlier chunks' histograms: the block's threads split the
  // chunks (thread i sums chunks i / E, i / E + parts, ...), then add up
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    base[e] = 0;
    rr_mod[e] = (int)(((rr[e] % nrep[e]) + nrep[e]) % nrep[e]);  // >= 0 for any rr
  }
  __syncthreads();
  {
    const int parts = blockDim.x / E > 0 ? blockDim.x / E : 1;
    for (int i = threadIdx.x; i < parts * E; i += blockDim.x) {
      const int e = i % E, part = i / E;
      int b = 0;
      for (int c = part; c < chunk; c += parts) b += chunk_hist[(int64_t)c * E + e];
      if (b) atomicAdd(&base[e], b);  // integer sums: the order does not matter
    }
  }
  for (int e = threadIdx.x; e < E; e += blockDim.x)
    for (int w = 0; w < kRouteWarps; ++w) wcnt[w][e] = 0;
  __syncthreads();
  // this warp's entries: tokens [t0, t0+32) -> flat entries [t0*k, (t0+32)*k)
  const int64_t t0 = (int64_t)chunk * kRouteChunkTokens + wp * 32;
  const int64_t f0 = t0 * k;
  for (int r = 0; r < k; ++r) {
    const int e = entry_expert(idx, valid, f0 + r * 32 + lane, k, n, E, nullptr);
    if (e >= 0) atomicAdd(&wcnt[wp][e], 1);
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    int run = 0;
    for (int w = 0; w < kRouteWarps; ++w) {
      wbase[w][e] = run;
      run += wcnt[w][e];
      wcnt[w][e] = 0;  // reused as the running count of pass 2
    }
  }
  __syncthreads();
  const unsigned lt_mask = (1u << lane) - 1u;
  for (int r = 0; r < k; ++r) {
    const int64_t f = f0 + r * 32 + lane;
    const int e = entry_expert(idx, valid, f, k, n, E, nullptr);
    const unsigned peers = __match_any_sync(0xffffffffu, e);
    const int rank_in_round = __popc(peers & lt_mask);
    int dest = -1, grp = 0;
    if (e >= 0) {
      const int within = base[e] + wbase[wp][e] + wcnt[wp][e] + rank_in_round;
      const int nr = nrep[e];
      const int slot = (rr_mod[e] + within) % nr;
      dest = owners[e * kMaxWorld + slot];
      grp = within / nr;
    }
    __syncwarp();
    if (e >= 0 && rank_in_round == 0) wcnt[wp][e] += __popc(peers);
    __syncwarp();
    if (f < n * k) {
      ent_dest[f] = dest;
      ent_grp[f] = grp;
    }
  }
}

// Round-robin state after a destination scan (mep_dest_ranks): rr[e] +=
// count[e], except on a layer without any replicated expert, whose state the
// reference's fast path (ep.py:84-85) leaves alone.
__global__ void __launch_bounds__(256) k_route_rr_advance(int nchunks, int E,
                                                          const int32_t* __restrict__ nrep,
                                                          int64_t* __restrict__ rr,
                                                          const int32_t* __restrict__ chunk_hist) {
  __shared__ int any_rep;
  if (threadIdx.x == 0) any_rep = 0;
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x)
    if (nrep[e] > 1) any_rep = 1;
  __syncthreads();
  if (!any_rep) return;
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    int c = 0;
    for (int ch = 0; ch < nchunks; ++ch) c += chunk_hist[(int64_t)ch * E + e];
    rr[e] += c;
  }
}

// Receive layout, send offsets and return-buffer tables from the exchanged
// counts C[s][d][e], by one CTA (256 threads), once every rank's counts for
// step `step` have arrived (bounded wait). Csm: world * world * E ints of
// shared memory for C.
//   receive side (this rank as owner d = rank): expert segments in
//     increasing expert order, each padded to kRowAlign rows, sources in rank
//     order inside a segment;
//   send side: dst_off[d][e] = the row of rank d's segment of e where this
//     rank's rows start;
//   return side: this rank's expert outputs come back in (owner d, expert e,
//     group index) order, group (d, e) starting at ret_off[d][e]; as an owner,
//     segment j's rows from source s start at src_begin[j][s] inside the
//     segment and belong at row ret_row[j][s] of s's return buffer.
__device__ void layout_block(int world, int rank, int E, const int32_t* __restrict__ owners,
                             const int32_t* __restrict__ nrep, const int32_t* cnt_in,
                             const uint32_t* flags, int64_t* __restrict__ recv_per_layer,
                             int64_t cap_rows, Layout* __restrict__ lay, uint32_t step,
                             const WaitCfg& wc, int* Csm) {
  __shared__ int R[kMaxWorld][kMaxExperts];       // rows per (dest, expert)
  __shared__ int before[kMaxWorld][kMaxExperts];  // rows from sources < rank
  __shared__ int seg[kMaxWorld][kMaxExperts];
  __shared__ unsigned char res[kMaxWorld][kMaxExperts];
  __shared__ int jof[kMaxExperts];                // local segment of expert e, or -1
  __shared__ int overflow[kMaxWorld];
  const int wp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int WE = world * E;
  if (threadIdx.x < world) wait_flag(flags + threadIdx.x, step, kErrWaitCounts, wc);
  __syncthreads();
  // peers stored the counts over NVLink: read them at L2 (not a stale L1 line)
  for (int i = threadIdx.x; i < world * WE; i += blockDim.x) Csm[i] = __ldcg(cnt_in + i);
  __syncthreads();
  for (int i = threadIdx.x; i < WE; i += blockDim.x) {
    const int d = i / E, e = i % E;
    int tot = 0, bef = 0;
    for (int s = 0; s < world; ++s) {
      const int c = Csm[s * WE + i];
      tot += c;
      if (s < rank) bef += c;
    }
    R[d][e] = tot;
    before[d][e] = bef;
    unsigned char r = 0;
    for (int j = 0; j < nrep[e]; ++j) r |= owners[e * kMaxWorld + j] == d;
    res[d][e] = r;
    if (tot > 0 && !r) set_err(wc.err, kErrNotResident);
  }
  __syncthreads();
  // warp d: padded segment bases at destination d (a scan over experts)
  if (wp < world) {
    const int d = wp;
    int run = 0;
    for (int e0 = 0; e0 < E; e0 += 32) {
      const int e = e0 + lane;
      const int v = (e < E && res[d][e]) ? (R[d][e] + kRowAlign - 1) / kRowAlign * kRowAlign : 0;
      const int inc = warp_inclusive_scan(v, lane);
      if (e < E) seg[d][e] = run + inc - v;
      run += __shfl_sync(0xffffffffu, inc, 31);
    }
    if (lane == 0) {
      overflow[d] = run > cap_rows;
      if (run > cap_rows) set_err(wc.err, kErrCapacity);
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < WE; i += blockDim.x) {
    const int d = i / E, e = i % E;
    lay->dst_off[d * kMaxExperts + e] = overflow[d] ? -1 : seg[d][e] + before[d][e];
  }
  // warp 0: this rank's local segments (scans over the resident experts)
  if (wp == 0) {
    int jrun = 0, trun = 0, rows = 0, end = 0;
    for (int e0 = 0; e0 < E; e0 += 32) {
      const int e = e0 + lane;
      const int mine = e < E && res[rank][e];
      const int rws = mine ? R[rank][e] : 0;
      const int t = (rws + kRowAlign - 1) / kRowAlign;
      const int jin = warp_inclusive_scan(mine, lane);
      const int tin = warp_inclusive_scan(t, lane);
      const int rin = warp_inclusive_scan(rws, lane);
      if (e < E) jof[e] = mine ? jrun + jin - 1 : -1;
      if (mine) {
        const int j = jrun + jin - 1;
        lay->local_expert[j] = e;
        lay->seg_base[j] = seg[rank][e];
        lay->seg_rows[j] = rws;
        lay->tile_prefix[j] = trun + tin - t;
        end = seg[rank][e] + t * kRowAlign;  // the last resident expert's lane holds the end
      }
      jrun += __shfl_sync(0xffffffffu, jin, 31);
      trun += __shfl_sync(0xffffffffu, tin, 31);
      rows += __shfl_sync(0xffffffffu, rin, 31);
      // the end of the last segment so far: the highest lane that holds one
      const unsigned has = __ballot_sync(0xffffffffu, mine);
      if (has) end = __shfl_sync(0xffffffffu, end, 31 - __clz(has));
    }
    if (lane == 0) {
      lay->tile_prefix[jrun] = trun;
      lay->n_local = jrun;
      lay->total_mtiles = overflow[rank] ? 0 : trun;
      lay->total_rows = end;
      lay->recv_rows = rows;
      if (recv_per_layer) recv_per_layer[0] += rows;
    }
  }
  __syncthreads();
  // warp s: running row offset of source s's return buffer over (owner d,
  // expert e) in order; its own buffer's group starts (s == rank), and where
  // the rows it sent this rank go (d == rank)
  if (wp < world) {
    const int src = wp;
    int run = 0;
    for (int d = 0; d < world; ++d) {
      for (int e0 = 0; e0 < E; e0 += 32) {
        const int e = e0 + lane;
        const int v = e < E ? Csm[src * WE + d * E + e] : 0;
        const int inc = warp_inclusive_scan(v, lane);
        const int excl = run + inc - v;
        if (e < E) {
          if (src == rank) lay->ret_off[d * kMaxExperts + e] = excl;
          if (d == rank && jof[e] >= 0) lay->ret_row[jof[e] * kMaxWorld + src] = excl;
        }
        run += __shfl_sync(0xffffffffu, inc, 31);
      }
    }
  }
  // per local segment: where each source's rows start inside it
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    const int j = jof[e];
    if (j < 0) continue;
    int run = 0;
    for (int src = 0; src < world; ++src) {
      lay->src_begin[j * (kMaxWorld + 1) + src] = run;
      run += Csm[src * WE + rank * E + e];
    }
    lay->src_begin[j * (kMaxWorld + 1) + world] = run;
  }
}

// ---------------------------------------------------------------------------
// The routing passes as ONE launch, for the layer step (the two-kernel scan
// above serves the stand-alone destination scan, mep_dest_ranks).
//
// grid G <= number of SMs (one 256-thread CTA per SM at most, so every CTA of
// the grid is resident at once); CTA b owns tokens [b*tpc, (b+1)*tpc), tpc a
// multiple of 256. Phase 1: every CTA reads the round-robin state, counts its
// kept entries per expert into chunk_hist[b] and arrives at a grid barrier
// (bounded wait). Phase 2: CTA 0 does the finalize work (totals, per-(dest,
// expert) counts, rr update after every CTA has read rr, stats, publish);
// every CTA then ranks its entries, 256 tokens per round, exactly as
// k_route_rank does for a chunk.
struct RouteSync {
  unsigned int count, gen;
};

__device__ __forceinline__ bool grid_barrier(RouteSync* gs, unsigned nblocks, const WaitCfg& wc) {
  __shared__ int ok;
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned g0 = *(volatile unsigned*)&gs->gen;  // read before arriving
    __threadfence();
    const unsigned prev = atomicAdd(&gs->count, 1u);
    if (prev == nblocks - 1) {
      gs->count = 0;  // every CTA has arrived: reset for the next launch, then release
      __threadfence();
      atomicAdd(&gs->gen, 1u);
      ok = 1;
    } else {
      ok = 1;
      const unsigned long long t0 = globaltimer_ns();
      for (uint32_t it = 0; *(volatile unsigned*)&gs->gen == g0; ++it) {
        __nanosleep(32);
        if ((it & 255u) == 255u && globaltimer_ns() - t0 > wc.timeout_ns) {
          set_err(wc.err, kErrPipeline);
          ok = 0;
          break;
        }
      }
    }
    __threadfence();
  }
  __syncthreads();
  return ok != 0;
}

static_assert(kMaxExperts <= 128, "the ranking keeps expert ids as int8");

__global__ void __launch_bounds__(kRouteThreads) k_route_fused(
    int64_t n, int k, int E, int64_t tpc, int world, int rank, const int64_t* __restrict__ idx,
    const uint8_t* __restrict__ valid, const int32_t* __restrict__ owners,
    const int32_t* __restrict__ nrep, int64_t* __restrict__ rr, int64_t* __restrict__ route_counts,
    int32_t* __restrict__ chunk_hist, int32_t* __restrict__ ent_dest,
    int32_t* __restrict__ ent_grp, int32_t* __restrict__ my_counts, PeerPtrs peers, uint32_t* seq,
    RouteSync* gs, const int32_t* cnt_in, const uint32_t* flags, int64_t* recv_per_layer,
    int64_t cap_rows, Layout* lay, WaitCfg wc, uint64_t* tl) {
  __shared__ int hist[kMaxExperts];
  __shared__ int base[kMaxExperts];   // entries of expert e before this CTA's range, then running
  __shared__ int tot[kMaxExperts];
  __shared__ int rr_mod[kMaxExperts];
  __shared__ int wcnt[kRouteWarps][kMaxExperts];
  __shared__ int wbase[kRouteWarps][kMaxExperts];
  __shared__ int8_t s_ev[kRouteWarps][kMaxTopk][32];  // a round's entries: expert id or -1
  __shared__ int cnt[kMaxWorld * kMaxExperts];
  __shared__ int s_nrep[kMaxExperts];
  __shared__ int s_own[kMaxExperts * kMaxWorld];
  __shared__ int any_rep;
  const int wp = warp_id(), lane = lane_id();
  const int b = blockIdx.x;
  // the last CTA has no tokens: it publishes the counts and lays out the
  // receive side while the others rank their entries
  const bool finalizer = b == (int)gridDim.x - 1;
  const int64_t t_beg = min((int64_t)b * tpc, n), t_end = min(t_beg + tpc, n);
  tl_begin(tl, kTlRoute);

  // ---- phase 1: round-robin state (read before anyone updates it), local histogram
  if (threadIdx.x == 0) any_rep = 0;
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    hist[e] = 0;
    base[e] = 0;
    tot[e] = 0;
    const int nr = nrep[e];
    s_nrep[e] = nr;
    rr_mod[e] = (int)(((rr[e] % nr) + nr) % nr);  // >= 0 for any rr
  }
  for (int i = threadIdx.x; i < E * kMaxWorld; i += blockDim.x) s_own[i] = owners[i];
  for (int i = threadIdx.x; i < kRouteWarps * kMaxExperts; i += blockDim.x) (&wcnt[0][0])[i] = 0;
  __syncthreads();
  // per-warp counters, and lanes holding the same expert add once: no
  // atomics (skewed routing piles entries on a few experts); each thread
  // keeps kRoutePrefetch loads in flight
  const unsigned lt_mask = (1u << lane) - 1u;
  for (int64_t f0 = t_beg * k; f0 < t_end * k; f0 += (int64_t)blockDim.x * kRoutePrefetch) {
    int ev[kRoutePrefetch];
#pragma unroll
    for (int j = 0; j < kRoutePrefetch; ++j) {
      const int64_t f = f0 + (int64_t)j * blockDim.x + threadIdx.x;
      ev[j] = f < t_end * k ? entry_expert(idx, valid, f, k, n, E, wc.err) : -1;
    }
#pragma unroll
    for (int j = 0; j < kRoutePrefetch; ++j) {
      const unsigned same = __match_any_sync(0xffffffffu, ev[j]);
      if (ev[j] >= 0 && (same & lt_mask) == 0) wcnt[wp][ev[j]] += __popc(same);
    }
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    int c = 0;
    for (int w = 0; w < kRouteWarps; ++w) c += wcnt[w][e];
    hist[e] = c;
    chunk_hist[(int64_t)b * E + e] = c;
  }
  tl_end(tl, kTlRouteHist);
  if (!grid_barrier(gs, gridDim.x, wc)) {
    // the barrier timed out (error word set): another CTA's histogram may be
    // missing, so this CTA routes nothing and leaves the round-robin state,
    // the statistics and the published counts untouched (the peers' bounded
    // waits then report the step as failed)
    for (int64_t f = t_beg * k + threadIdx.x; f < t_end * k; f += blockDim.x) ent_dest[f] = -1;
    tl_end(tl, kTlRoute + 1);
    return;
  }

  // ---- phase 2: prefix of the earlier CTAs' counts and the totals
  {
    const int parts = blockDim.x / E > 0 ? blockDim.x / E : 1;
    const int G = (int)gridDim.x;
    for (int i = threadIdx.x; i < parts * E; i += blockDim.x) {
      const int e = i % E, part = i / E;
      int bsum = 0, tsum = 0;
      for (int c0 = part; c0 < G; c0 += parts * kRoutePrefetch) {
        int v[kRoutePrefetch];
#pragma unroll
        for (int j = 0; j < kRoutePrefetch; ++j) {
          const int c = c0 + j * parts;
          v[j] = c < G ? __ldcg(chunk_hist + (int64_t)c * E + e) : 0;
        }
#pragma unroll
        for (int j = 0; j < kRoutePrefetch; ++j) {
          tsum += v[j];
          if (c0 + j * parts < b) bsum += v[j];
        }
      }
      if (bsum) atomicAdd(&base[e], bsum);
      if (tsum) atomicAdd(&tot[e], tsum);
    }
  }
  __syncthreads();

  if (finalizer) {
    if (threadIdx.x == 0) tl_mark(tl, kTlRouteSync);
    // finalize: counts per (dest, expert), rr, stats, publish
    const uint32_t step = *seq + 1u;
    for (int i = threadIdx.x; i < world * E; i += blockDim.x) cnt[i] = 0;
    for (int e = threadIdx.x; e < E; e += blockDim.x)
      if (s_nrep[e] > 1) any_rep = 1;
    __syncthreads();
    for (int e = threadIdx.x; e < E; e += blockDim.x) {
      const int c = tot[e];
      const int nr = s_nrep[e];
      const int rr0 = rr_mod[e];
      for (int j = 0; j < nr; ++j) {
        const int d = s_own[e * kMaxWorld + j];
        const int w0 = ((j - rr0) % nr + nr) % nr;
        cnt[d * E + e] = c > w0 ? (c - w0 - 1) / nr + 1 : 0;
      }
    }
    __syncthreads();
    // publish first (the peers wait for it), then the local bookkeeping
    for (int d = 0; d < world; ++d) {
      int32_t* dst = peers.cnt_in[d] + (int64_t)rank * world * E;
      for (int i = threadIdx.x; i < world * E; i += blockDim.x) dst[i] = cnt[i];
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      fence_acq_rel_sys();  // every thread's count stores (ordered by the barrier) before the flags
      for (int d = 0; d < world; ++d) st_relaxed_sys(peers.flags[d] + rank, step);
      *seq = step;
      tl_mark(tl, kTlCountsSent);
    }
    for (int i = threadIdx.x; i < world * E; i += blockDim.x) my_counts[i] = cnt[i];
    for (int e = threadIdx.x; e < E; e += blockDim.x) {
      if (any_rep) rr[e] += tot[e];
      if (route_counts) route_counts[e] += tot[e];
    }
    // the receive layout, once every rank's counts are in
    extern __shared__ int route_dyn[];  // world * world * E counts for the layout pass
    layout_block(world, rank, E, s_own, s_nrep, cnt_in, flags, recv_per_layer, cap_rows, lay,
                 step, wc, route_dyn);
    __syncthreads();
    if (threadIdx.x == 0) tl_mark(tl, kTlLayout);
  }

  // ---- ranking, 256 tokens per round (8 warps x 32 tokens)
  for (int64_t r0 = t_beg; r0 < t_end; r0 += kRouteChunkTokens) {
    for (int e = threadIdx.x; e < E; e += blockDim.x)
      for (int w = 0; w < kRouteWarps; ++w) wcnt[w][e] = 0;
    __syncthreads();
    const int64_t t0 = r0 + wp * 32;
    const int64_t f0 = t0 * k;
    const int64_t f_end = min(r0 + kRouteChunkTokens, t_end) * k;
    // this warp's entries of the round, loaded once for both passes into
    // shared memory. The loops stay rolled: each CTA runs them once or a few
    // times, so their time is the instruction fetch of their code, not its
    // issue.
#pragma unroll 1
    for (int r = 0; r < k; ++r) {
      const int64_t f = f0 + r * 32 + lane;
      s_ev[wp][r][lane] = f < f_end ? entry_expert(idx, valid, f, k, n, E, nullptr) : -1;
    }
    __syncwarp();
#pragma unroll 1
    for (int r = 0; r < k; ++r) {
      const int e = s_ev[wp][r][lane];
      const unsigned same = __match_any_sync(0xffffffffu, e);
      if (e >= 0 && (same & lt_mask) == 0) wcnt[wp][e] += __popc(same);
    }
    __syncthreads();
    for (int e = threadIdx.x; e < E; e += blockDim.x) {
      int run = 0;
      for (int w = 0; w < kRouteWarps; ++w) {
        wbase[w][e] = run;
        run += wcnt[w][e];
        wcnt[w][e] = 0;  // reused as the running count of the pass below
      }
      hist[e] = run;  // this round's total, added to base after the pass
    }
    __syncthreads();
#pragma unroll 1
    for (int r = 0; r < k; ++r) {
      const int64_t f = f0 + r * 32 + lane;
      const int e = s_ev[wp][r][lane];
      const unsigned peers_mask = __match_any_sync(0xffffffffu, e);
      const int rank_in_round = __popc(peers_mask & lt_mask);
      int dest = -1, grp = 0;
      if (e >= 0) {
        const int within = base[e] + wbase[wp][e] + wcnt[wp][e] + rank_in_round;
        const int nr = s_nrep[e];
        int slot = 0;
        grp = within;
        if (nr > 1) {  // a replicated expert: round-robin over its owners
          slot = (rr_mod[e] + within) % nr;
          grp = within / nr;
        }
        dest = s_own[e * kMaxWorld + slot];
      }
      __syncwarp();
      if (e >= 0 && rank_in_round == 0) wcnt[wp][e] += __popc(peers_mask);
      __syncwarp();
      if (f < f_end) {
        ent_dest[f] = dest;
        ent_grp[f] = grp;
      }
    }
    __syncthreads();
    for (int e = threadIdx.x; e < E; e += blockDim.x) base[e] += hist[e];
    __syncthreads();
  }
  tl_end(tl, kTlRoute + 1);
}

__global__ void k_dest_to_i64(int64_t m, const int32_t* __restrict__ d, int64_t* __restrict__ out) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < m) out[i] = d[i];
}

}  // namespace

void launch_route(int64_t n, int topk, int experts, int world, int rank,
                  const int64_t* topk_idx, const uint8_t* valid, const int32_t* owners_l,
                  const int32_t* nrep_l, int64_t* rr_l, int64_t* route_counts_l,
                  int32_t* chunk_hist, int32_t* ent_dest, int32_t* ent_grp, int32_t* my_counts,
                  const PeerPtrs& peers, uint32_t* seq, unsigned int* sync, int num_sms,
                  const int32_t* cnt_in_local, const uint32_t* flags_local,
                  int64_t* recv_per_layer_l, int64_t cap_rows, Layout* layout, WaitCfg wc,
                  uint64_t* tl, cudaStream_t st) {
  // one CTA per 256-token round, at most one per SM (all resident for the
  // grid barrier), plus the finalizing CTA
  const int64_t rounds = (n + kRouteChunkTokens - 1) / kRouteChunkTokens;
  int64_t chunks = rounds < num_sms - 1 ? rounds : num_sms - 1;
  if (chunks < 1) chunks = 1;
  const int64_t grid = chunks + 1;
  const int64_t tpc = (rounds + chunks - 1) / chunks * kRouteChunkTokens;
  const size_t dyn = (size_t)world * world * experts * sizeof(int);  // <= 32 KiB
  static size_t dyn_set = 0;
  if (dyn > dyn_set) {
    cudaFuncSetAttribute(k_route_fused, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)dyn);
    dyn_set = dyn;
  }
  k_route_fused<<<(unsigned)grid, kRouteThreads, dyn, st>>>(
      n, topk, experts, tpc, world, rank, topk_idx, valid, owners_l, nrep_l, rr_l, route_counts_l,
      chunk_hist, ent_dest, ent_grp, my_counts, peers, seq, reinterpret_cast<RouteSync*>(sync),
      cnt_in_local, flags_local, recv_per_layer_l, cap_rows, layout, wc, tl);
}

void launch_dest_only(int64_t m, int experts, const int64_t* expert_ids, const int32_t* owners_l,
                      const int32_t* nrep_l, int64_t* rr_l, int32_t* chunk_hist,
                      int32_t* ent_dest, int32_t* ent_grp, int64_t* dest_out, WaitCfg wc,
                      cudaStream_t st) {
  const int nchunks = (int)((m + kRouteChunkTokens - 1) / kRouteChunkTokens);
  if (nchunks > 0) {
    k_route_hist<<<nchunks, kRouteThreads, 0, st>>>(m, 1, experts, expert_ids, nullptr, chunk_hist,
                                                    wc.err);
    k_route_rank<<<nchunks, kRouteThreads, 0, st>>>(m, 1, experts, expert_ids, nullptr, owners_l,
                                                    nrep_l, rr_l, chunk_hist, ent_dest, ent_grp);
    k_dest_to_i64<<<(unsigned)((m + 255) / 256), 256, 0, st>>>(m, ent_dest, dest_out);
  }
  k_route_rr_advance<<<1, 256, 0, st>>>(nchunks, experts, nrep_l, rr_l, chunk_hist);
}


}  // namespace mep
