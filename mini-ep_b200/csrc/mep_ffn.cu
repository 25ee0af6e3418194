// Expert FFN over the expert-grouped receive buffer (run_experts,
// miniep/modeling.py:83-104):
//     h   = x_e @ w_in[e]^T            (rounded to the model dtype)
//     act = silu(h[:, :I]) * h[:, I:]  (each op rounded to the model dtype)
//     y   = act @ w_out[e]^T           (rounded), stored straight back to the
//                                      source rank's (token, slot) landing row.
//
// Two implementations share the tile schedule (Layout: expert segments padded
// to 128 rows, tile t -> (segment, row tile, N block)):
//   * tcgen05 (bf16): persistent, warp-specialised kernel. Warp 0 issues TMA
//     loads (128B-swizzled K-major tiles) into a shared-memory stage ring,
//     warp 1 issues tcgen05.mma (N=256, K=16) into a double-buffered TMEM
//     accumulator (2 x 256 columns), warps 2-9 drain TMEM with tcgen05.ld and
//     run the epilogue (SwiGLU, or the store to the source rank's landing
//     buffer over NVLink) while the next tile accumulates. By default a pair
//     of CTAs (2-CTA cluster, tcgen05.mma.cta_group::2) computes a 256x256
//     tile; the single-CTA 128x256 variant stays selectable.
//     GEMM1 puts the gate rows [n, n+128) and the up rows [I+n, I+n+128) of
//     w_in side by side in one 256-row B tile, so one MMA chain produces both
//     halves of the SwiGLU for the same rows.
//   * CUDA cores (fp32, and bf16 when asked): 64x64 register-tiled FMA kernel.
#include <cstdint>
#include <cstring>
#include <cuda.h>
#include <cudaTypedefs.h>
#include "mep_device.cuh"
#include "mep_tc.cuh"

namespace mep {
namespace {

using bf16 = __nv_bfloat16;

__device__ __forceinline__ void grid_done_signal_ffn(unsigned int* done_ctr, const PeerPtrs& peers,
                                                     int world, int rank, const uint32_t* seq) {
  if (world == 1) return;  // one rank: the combine follows in stream order
  __syncthreads();  // this CTA's stores happen before thread 0's fence below
  if (threadIdx.x == 0) {
    fence_acq_rel_sys();
    const unsigned prev = atomicAdd(done_ctr, 1u);
    if (prev == gridDim.x - 1) {
      fence_acq_rel_sys();
      const uint32_t step = *seq;
      for (int d = 0; d < world; ++d) st_relaxed_sys(peers.flags[d] + 2 * world + rank, step);
      *done_ctr = 0u;
    }
  }
}

// Tile t of a schedule with `ntiles_n` N-blocks and `sub` row-blocks per
// 128-row tile -> local expert j, first padded row, rows left in the segment
// from that row, N-block.
struct TileCoord {
  int j, row0, rows, nb;
};
__device__ __forceinline__ TileCoord decode_tile(int t, int ntiles_n, int sub, int sub_rows,
                                                 int tile_rows, int n_local,
                                                 const int* tile_prefix, const int* seg_base,
                                                 const int* seg_rows) {
  TileCoord c;
  const int mt = t / ntiles_n;
  c.nb = t - mt * ntiles_n;
  const int mtile = mt / sub;
  const int part = mt - mtile * sub;
  int j = 0;
  while (j + 1 < n_local && tile_prefix[j + 1] <= mtile) ++j;
  c.j = j;
  const int local_row = (mtile - tile_prefix[j]) * tile_rows + part * sub_rows;
  c.row0 = seg_base[j] + local_row;
  c.rows = seg_rows[j] - local_row;
  return c;
}

__device__ __forceinline__ float silu_mul(float g, float u, bool is_bf16) {
  // gate and up are rounded to the model dtype, then silu(gate) and the
  // product are each rounded to it (the caller rounds the product)
  if (is_bf16) {
    const float gr = __bfloat162float(__float2bfloat16_rn(g));
    const float ur = __bfloat162float(__float2bfloat16_rn(u));
    const float s = __bfloat162float(__float2bfloat16_rn(gr / (1.f + expf(-gr))));
    return s * ur;
  }
  return (g / (1.f + expf(-g))) * u;
}

// ===================================================================== SIMT
constexpr int kSimtBM = 64, kSimtBN = 64, kSimtBK = 16;

template <typename T, int MODE>
__global__ void __launch_bounds__(256) k_ffn_simt(const T* __restrict__ A, int lda,
                                                  const T* __restrict__ B, int K,
                                                  int b_rows_per_expert, int b_up_off,
                                                  int ntiles_n, const Layout* __restrict__ lay,
                                                  T* __restrict__ act, int act_ld,
                                                  PeerPtrs peers,
                                                  int H, int world, int rank,
                                                  unsigned int* done_ctr, const uint32_t* seq,
                                                  uint64_t* tl) {
  __shared__ float As[kSimtBK][kSimtBM + 4];
  tl_begin(tl, MODE == 0 ? kTlGemm1 : kTlGemm2);
  __shared__ float Bs[kSimtBK][kSimtBN + 4];
  __shared__ float Cs[kSimtBM][kSimtBN + 1];
  __shared__ int s_prefix[kMaxExperts + 1], s_base[kMaxExperts], s_rows[kMaxExperts];
  const int n_local = lay->n_local;
  for (int i = threadIdx.x; i <= n_local; i += blockDim.x) s_prefix[i] = lay->tile_prefix[i];
  for (int i = threadIdx.x; i < n_local; i += blockDim.x) {
    s_base[i] = lay->seg_base[i];
    s_rows[i] = lay->seg_rows[i];
  }
  __syncthreads();
  const int total = lay->total_mtiles * 2 * ntiles_n;
  const int tid = threadIdx.x, ty = tid >> 4, tx = tid & 15;
  for (int t = blockIdx.x; t < total; t += gridDim.x) {
    const TileCoord c = decode_tile(t, ntiles_n, 2, kSimtBM, kRowAlign, n_local, s_prefix, s_base, s_rows);
    if (c.rows <= 0) continue;  // second half of a partly filled 128-row tile
    // B rows of this tile: MODE 0 -> 32 gate rows then 32 up rows; MODE 1 -> 64 rows
    const int64_t bexp = (int64_t)c.j * b_rows_per_expert;
    float acc[4][4] = {};
    for (int k0 = 0; k0 < K; k0 += kSimtBK) {
      for (int i = tid; i < kSimtBM * kSimtBK; i += 256) {
        const int r = i / kSimtBK, kk = i % kSimtBK;
        As[kk][r] = Elt<T>::to_f(A[(int64_t)(c.row0 + r) * lda + k0 + kk]);
        int64_t brow;
        if (MODE == 0)
          brow = bexp + (r < 32 ? c.nb * 32 + r : b_up_off + c.nb * 32 + (r - 32));
        else
          brow = bexp + c.nb * kSimtBN + r;
        Bs[kk][r] = Elt<T>::to_f(B[brow * K + k0 + kk]);
      }
      __syncthreads();
#pragma unroll
      for (int kk = 0; kk < kSimtBK; ++kk) {
        float a[4], b[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) a[i] = As[kk][ty * 4 + i];
#pragma unroll
        for (int j = 0; j < 4; ++j) b[j] = Bs[kk][tx * 4 + j];
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
      }
      __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) Cs[ty * 4 + i][tx * 4 + j] = acc[i][j];
    __syncthreads();
    if (MODE == 0) {
      for (int i = tid; i < kSimtBM * 32; i += 256) {
        const int r = i / 32, cc = i % 32;
        if (r < c.rows) {
          const float a = silu_mul(Cs[r][cc], Cs[r][32 + cc], sizeof(T) == 2);
          act[(int64_t)(c.row0 + r) * act_ld + c.nb * 32 + cc] = Elt<T>::from_f(a);
        }
      }
    } else {
      // row -> (source rank, row of its return buffer)
      const int* sb = lay->src_begin + c.j * (kMaxWorld + 1);
      const int* rr = lay->ret_row + c.j * kMaxWorld;
      for (int i = tid; i < kSimtBM * kSimtBN; i += 256) {
        const int r = i / kSimtBN, cc = i % kSimtBN;
        if (r < c.rows) {
          const int lr = c.row0 - s_base[c.j] + r;
          int src = 0;
          while (src + 1 < world && sb[src + 1] <= lr) ++src;
          T* dst = static_cast<T*>(peers.ret[src]) + (int64_t)(rr[src] + lr - sb[src]) * H;
          dst[c.nb * kSimtBN + cc] = Elt<T>::from_f(Cs[r][cc]);
        }
      }
    }
    __syncthreads();
  }
  if (MODE == 1) grid_done_signal_ffn(done_ctr, peers, world, rank, seq);
  tl_end(tl, (MODE == 0 ? kTlGemm1 : kTlGemm2) + 1);
}

// =================================================================== tcgen05
namespace ffn {
using namespace ::mep::tc;  // the shared tcgen05 / TMA building blocks (mep_tc.cuh)
constexpr int BN = 256, BK = 64;
constexpr int A_TILE = 128 * BK * 2;            // 16 KiB: 128 rows x 64 bf16 (one 128B-swizzle row each)
constexpr int EPI_WARPS = 8;                    // two per TMEM lane quadrant, splitting the columns
constexpr int THREADS = 64 + 32 * EPI_WARPS;    // warp0 TMA, warp1 MMA, warps 2-9 epilogue
constexpr int TMEM_COLS = 512;                  // two 256-column fp32 accumulators
constexpr unsigned long long kWaitNs = 2000000000ull;  // bounded mbarrier waits (2 s)

// Per-variant geometry. Single CTA: a 128x256 tile per CTA, the CTA loads
// 128 A rows + 256 B rows per k-block. CTA pair: a 256x256 tile per 2-CTA
// cluster, each CTA loads its 128 A rows + 128 of the B rows.
// A-stationary (AST, CTA pairs, K <= 512): a pair works through all N blocks
// of one 256-row tile in a row; its A rows stay in shared memory (one slot
// per k-block) across them, and only B streams through the stage ring. The
// operands loaded per row tile drop from N blocks x (A + B) to A + N blocks
// x B (GEMM2 of shape (a): 640 KiB instead of 1 MiB per CTA), and the stage
// loads, not the tensor pipe, are what bound this kernel otherwise.
constexpr int AST_SLOTS = 8;  // resident A k-blocks: K <= 512
template <bool PAIR, bool AST = false>
struct Geo {
  static constexpr int TILE_M = PAIR ? 256 : 128;
  static constexpr int B_ROWS = PAIR ? 128 : 256;         // B rows held by one CTA
  static constexpr int A_REGION = AST ? AST_SLOTS * A_TILE : 0;
  static constexpr int STAGE = (AST ? 0 : A_TILE) + B_ROWS * BK * 2;  // bytes per stage per CTA
  static constexpr int STAGES = AST ? 4 : (PAIR ? 6 : 4);
  static constexpr int DATA = A_REGION + STAGES * STAGE;
  static constexpr uint32_t TX = (PAIR ? 2 : 1) * STAGE;  // bytes landing on the leader's barrier
  static constexpr uint32_t TX_A = (PAIR ? 2 : 1) * A_TILE;
  // kind::f16 instruction descriptor: D f32, A/B bf16, both K-major, N=256, M=TILE_M
  static constexpr uint32_t IDESC = (1u << 4) | (1u << 7) | (1u << 10) |
                                    ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(TILE_M >> 4) << 24);
  static constexpr uint32_t TEMPTY_ARRIVALS = EPI_WARPS * (PAIR ? 2 : 1);
};

template <bool PAIR, bool AST = false>
struct Smem {
  uint64_t full[Geo<PAIR, AST>::STAGES], empty[Geo<PAIR, AST>::STAGES], tfull[2], tempty[2];
  uint64_t a_full[AST_SLOTS], a_empty[AST_SLOTS];  // A-stationary: resident A slots
  uint32_t tmem_base;
  int abort;
  int n_local, total;
  int prefix[kMaxExperts + 1], base[kMaxExperts], rows[kMaxExperts];
};
// epilogue staging: 32 rows x 128 B per warp, 16-byte chunks XOR-swizzled by row
constexpr int STAGE_WARP_BYTES = 32 * 128;
template <bool PAIR, bool AST = false>
__host__ __device__ constexpr int off_stage() {  // 1024-aligned: TMA 128B-swizzle tile source
  return Geo<PAIR, AST>::DATA + (((int)sizeof(Smem<PAIR, AST>) + 1023) / 1024) * 1024;
}
template <bool PAIR, bool AST = false>
__host__ __device__ constexpr int smem_bytes() {
  return off_stage<PAIR, AST>() + EPI_WARPS * STAGE_WARP_BYTES + 1024;
}
static_assert(smem_bytes<false>() <= 232448, "single-CTA kernel exceeds shared memory");
static_assert(smem_bytes<true>() <= 232448, "CTA-pair kernel exceeds shared memory");
static_assert(smem_bytes<true, true>() <= 232448, "A-stationary kernel exceeds shared memory");

// Bounded wait: false (and the CTA abort flag + device error set) on timeout
// or when another role of this CTA already gave up.
template <class SM>
__device__ __forceinline__ bool mbar_wait(uint64_t* b, uint32_t parity, SM* S, int* err) {
  if (mbar_try(b, parity)) return true;
  const unsigned long long t0 = globaltimer_ns();
  for (uint32_t it = 0;; ++it) {
    if (mbar_try(b, parity)) return true;
    if ((it & 63u) == 63u) {
      if (*(volatile int*)&S->abort) return false;
      if (globaltimer_ns() - t0 > kWaitNs) {
        *(volatile int*)&S->abort = 1;
        set_err(err, kErrPipeline);
        return false;
      }
    }
  }
}
// silu(bf16(g)) rounded to bf16, times bf16(u): the rounding points of the
// reference's bf16 SwiGLU (modeling.py:102-103). The fp32 sigmoid uses the
// fast exponential and division intrinsics (a few fp32 ulp from the exact
// expressions, far inside one bf16 rounding step).
__device__ __forceinline__ float swiglu_bf16(float g, float u) {
  const float gr = bf16_round(g);
  const float s = bf16_round(__fdividef(gr, 1.f + __expf(-gr)));
  return s * bf16_round(u);
}

// Store this warp's 32 rows x 64 bf16 columns (128 B per row): lane l holds row
// l's 32 packed words in v and that row's destination in dst (nullptr = skip).
// The rows go through the warp's shared-memory slice (16-byte chunks
// XOR-swizzled by row, conflict-free both ways) so that every store
// instruction writes four whole 128-byte row segments (coalesced for HBM and
// for NVLink when the destination is a peer's buffer).
__device__ __forceinline__ void warp_store_rows(uint8_t* stage, const uint32_t (&v)[32],
                                                void* dst, int lane) {
  uint8_t* srow = stage + lane * 128;
#pragma unroll
  for (int i = 0; i < 8; ++i)
    *reinterpret_cast<uint4*>(srow + ((i ^ (lane & 7)) << 4)) =
        make_uint4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
  __syncwarp();
  const unsigned long long mine = reinterpret_cast<unsigned long long>(dst);
#pragma unroll
  for (int it = 0; it < 8; ++it) {
    const int r = it * 4 + (lane >> 3), seg = lane & 7;
    const unsigned long long d = __shfl_sync(0xffffffffu, mine, r);
    const uint4 val = *reinterpret_cast<const uint4*>(stage + r * 128 + ((seg ^ (r & 7)) << 4));
    if (d) reinterpret_cast<uint4*>(d)[seg] = val;
  }
  __syncwarp();
}

// Tensor maps of every rank's return buffer (rows of H bf16, boxes of 32
// rows x 64 columns, 128B swizzle): GEMM2's tile stores
struct RetMaps {
  CUtensorMap m[kMaxWorld];
};

struct TcArgs {
  const Layout* lay;
  int K;                   // reduction length
  int ntiles_n;            // N blocks per row tile
  int b_rows_per_expert;   // rows of B per local expert (2I or H)
  int b_step;              // B rows advanced per N block (128 for GEMM1, 256 for GEMM2)
  int b_second;            // offset of the second 128-row half of the B tile
  bf16* act;               // MODE 0 output
  int act_ld;
  PeerPtrs peers;
  int H, world, rank;
  unsigned int* done_ctr;
  const uint32_t* seq;
  int* err;
  uint64_t* tl;            // step timeline or null
  int prefetch;            // 1: prefetch the unit's next tile's A rows into L2
};

// MODE 0: GEMM1 + SwiGLU -> act. MODE 1: GEMM2 -> source landing rows.
// PAIR: one 256-row tile per 2-CTA cluster with tcgen05.mma.cta_group::2.
// The i-th tile a unit (CTA or CTA pair) works on: units take tiles
// round-robin, or, A-stationary, whole row tiles (all their N blocks in order).
template <bool AST>
__device__ __forceinline__ int unit_tile(int i, int unit, int nunits, int ntiles_n) {
  if (!AST) return unit + i * nunits;
  return (unit + (i / ntiles_n) * nunits) * ntiles_n + i % ntiles_n;
}

template <int MODE, bool PAIR, bool AST = false>
__global__ void __launch_bounds__(THREADS, 1) k_ffn_tc(const __grid_constant__ CUtensorMap tmA,
                                                       const __grid_constant__ CUtensorMap tmB,
                                                       const __grid_constant__ RetMaps rmaps,
                                                       const TcArgs args) {
  using G = Geo<PAIR, AST>;
  using SM = Smem<PAIR, AST>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  SM* S = reinterpret_cast<SM*>(smem + G::DATA);
  uint8_t* ring = smem + G::A_REGION;  // the stage ring (after the resident A slots)
  const int wp = warp_id(), lane = lane_id();
  const uint32_t cta = PAIR ? cluster_rank() : 0u;
  const bool leader = cta == 0;
  tl_begin(args.tl, MODE == 0 ? kTlGemm1 : kTlGemm2);

  if (threadIdx.x == 32) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    if (MODE == 1)
      for (int r = 0; r < args.world; ++r) tma_prefetch_desc(&rmaps.m[r]);
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < G::STAGES; ++s) {
      mbar_init(&S->full[s], 1);
      mbar_init(&S->empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&S->tfull[b], 1);
      mbar_init(&S->tempty[b], G::TEMPTY_ARRIVALS);  // used in the leader
    }
    for (int a = 0; a < AST_SLOTS; ++a) {
      mbar_init(&S->a_full[a], 1);
      mbar_init(&S->a_empty[a], 1);
    }
    S->abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (wp == 1) {
    if (PAIR) {
      asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                       smem_u32(&S->tmem_base)),
                   "r"(TMEM_COLS)
                   : "memory");
      asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
    } else {
      asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                       smem_u32(&S->tmem_base)),
                   "r"(TMEM_COLS)
                   : "memory");
      asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
  }
  {
    // the local segments, loaded in parallel; warp 2 scans their row tiles
    // of TILE_M rows (one load round trip, not one per expert)
    const Layout* lay = args.lay;
    const int nl = lay->n_local;
    for (int i = threadIdx.x; i < nl; i += blockDim.x) {
      S->base[i] = lay->seg_base[i];
      S->rows[i] = lay->seg_rows[i];
    }
    if (wp == 2) {
      int run = 0;
      for (int j0 = 0; j0 < nl; j0 += 32) {
        const int j = j0 + lane;
        const int t = j < nl ? (lay->seg_rows[j] + G::TILE_M - 1) / G::TILE_M : 0;
        const int inc = warp_inclusive_scan(t, lane);
        if (j < nl) S->prefix[j] = run + inc - t;
        run += __shfl_sync(0xffffffffu, inc, 31);
      }
      if (lane == 0) {
        S->prefix[nl] = run;
        S->n_local = nl;
        S->total = lay->total_mtiles > 0 ? run * args.ntiles_n : 0;
      }
    }
  }
  fence_before();
  __syncthreads();
  if (PAIR) cluster_sync();  // the peer's barriers exist before any remote arrive or TMA completion
  fence_after();
  const uint32_t tmem_base = S->tmem_base;
  const int total = S->total;
  const int kblocks = args.K / BK;
  const int unit = PAIR ? (int)(blockIdx.x >> 1) : (int)blockIdx.x;
  const int nunits = PAIR ? (int)(gridDim.x >> 1) : (int)gridDim.x;

  if (wp == 0) {
    // ---------------------------------------------------------------- TMA producer
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0;
      for (int i = 0;; ++i) {
        const int t = unit_tile<AST>(i, unit, nunits, args.ntiles_n);
        if (t >= total) break;
        const TileCoord c = decode_tile(t, args.ntiles_n, 1, G::TILE_M, G::TILE_M, S->n_local,
                                        S->prefix, S->base, S->rows);
        const int arow = c.row0 + (int)cta * 128;
        const int brow = c.j * args.b_rows_per_expert + c.nb * args.b_step;
        const uint32_t a_ph = (uint32_t)(i / args.ntiles_n) & 1u;  // AST: row tiles so far
        // the rows of this unit's next tile, prefetched into L2 one k-block at a time
        int next_arow = -1;
        if (!AST && args.prefetch) {
          const int tn = unit_tile<AST>(i + 1, unit, nunits, args.ntiles_n);
          if (tn < total)
            next_arow = decode_tile(tn, args.ntiles_n, 1, G::TILE_M, G::TILE_M, S->n_local,
                                    S->prefix, S->base, S->rows).row0 + (int)cta * 128;
        }
        bool ok = true;
        for (int kb = 0; kb < kblocks; ++kb) {
          if (AST && c.nb == 0) {
            // A slot kb: free once the previous row tile's last N block used it
            if (!mbar_wait(&S->a_empty[kb], a_ph ^ 1u, S, args.err)) {
              ok = false;
              break;
            }
            if (leader) mbar_expect_tx(&S->a_full[kb], G::TX_A);
            const uint32_t abar = map_to_cta(&S->a_full[kb], 0);
            tma_load_2d<PAIR>(smem + kb * A_TILE, &tmA, kb * BK, arow, abar);
          }
          if (!mbar_wait(&S->empty[s], ph ^ 1u, S, args.err)) {
            ok = false;
            break;
          }
          if (leader) mbar_expect_tx(&S->full[s], G::TX);
          const uint32_t bar = PAIR ? map_to_cta(&S->full[s], 0) : smem_u32(&S->full[s]);
          uint8_t* st = ring + s * G::STAGE;
          if (AST) {
            tma_load_2d<PAIR>(st, &tmB, kb * BK, brow + (cta ? args.b_second : 0), bar);
          } else if (PAIR) {
            tma_load_2d<PAIR>(st, &tmA, kb * BK, arow, bar);
            tma_load_2d<PAIR>(st + A_TILE, &tmB, kb * BK, brow + (cta ? args.b_second : 0), bar);
          } else {
            tma_load_2d<PAIR>(st, &tmA, kb * BK, arow, bar);
            tma_load_2d<PAIR>(st + A_TILE, &tmB, kb * BK, brow, bar);
            tma_load_2d<PAIR>(st + A_TILE + A_TILE, &tmB, kb * BK, brow + args.b_second, bar);
          }
          if (next_arow >= 0) tma_prefetch_2d(&tmA, kb * BK, next_arow);
          if (++s == G::STAGES) {
            s = 0;
            ph ^= 1u;
          }
        }
        if (!ok) break;
      }
    }
  } else if (wp == 1) {
    // ---------------------------------------------------------------- MMA issuer (leader)
    if (leader && lane == 0) {
      int s = 0;
      uint32_t ph = 0;
      for (int it = 0;; ++it) {
        const int t = unit_tile<AST>(it, unit, nunits, args.ntiles_n);
        if (t >= total) break;
        const int nb = t % args.ntiles_n;
        const uint32_t a_ph = (uint32_t)(it / args.ntiles_n) & 1u;
        const int b = it & 1;
        const uint32_t aph = (uint32_t)(it >> 1) & 1u;
        if (!mbar_wait(&S->tempty[b], aph ^ 1u, S, args.err)) break;
        fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(b * BN);
        bool ok = true;
        for (int kb = 0; kb < kblocks; ++kb) {
          if (AST && nb == 0) {
            if (!mbar_wait(&S->a_full[kb], a_ph, S, args.err)) {
              ok = false;
              break;
            }
          }
          if (!mbar_wait(&S->full[s], ph, S, args.err)) {
            ok = false;
            break;
          }
          fence_after();
          const uint32_t a0 = AST ? smem_u32(smem + kb * A_TILE) : smem_u32(ring + s * G::STAGE);
          const uint32_t b0 = AST ? smem_u32(ring + s * G::STAGE) : a0 + A_TILE;
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk)
            mma_f16<PAIR>(d_tmem, sw128_desc(a0 + kk * 32), sw128_desc(b0 + kk * 32), G::IDESC,
                          (kb | kk) != 0);
          mma_commit<PAIR>(&S->empty[s]);
          // the row tile's last N block frees A slot kb for the next row tile
          if (AST && nb == args.ntiles_n - 1) mma_commit<PAIR>(&S->a_empty[kb]);
          if (++s == G::STAGES) {
            s = 0;
            ph ^= 1u;
          }
        }
        if (!ok) break;
        mma_commit<PAIR>(&S->tfull[b]);
      }
    }
  } else {
    // ---------------------------------------------------------------- epilogue
    // warp wp may read TMEM lanes [32*(wp%4), +32) only; the two warps of a
    // quadrant split the columns (h = 0, 1)
    const int e = wp - 2;
    const int q = wp & 3, h = e >> 2;
    const int m = q * 32 + lane;
    const uint32_t tempty_leader[2] = {PAIR ? map_to_cta(&S->tempty[0], 0) : smem_u32(&S->tempty[0]),
                                       PAIR ? map_to_cta(&S->tempty[1], 0) : smem_u32(&S->tempty[1])};
    uint8_t* stage = smem + off_stage<PAIR, AST>() + e * STAGE_WARP_BYTES;
    for (int it = 0;; ++it) {
      const int t = unit_tile<AST>(it, unit, nunits, args.ntiles_n);
      if (t >= total) break;
      const int b = it & 1;
      const uint32_t aph = (uint32_t)(it >> 1) & 1u;
      const TileCoord c = decode_tile(t, args.ntiles_n, 1, G::TILE_M, G::TILE_M, S->n_local,
                                      S->prefix, S->base, S->rows);
      const int r = (int)cta * 128 + m;  // row inside the tile
      const bool valid = r < c.rows;
      const int64_t grow = c.row0 + r;
      // MODE 1: this warp's 32 rows [lr0, lr0 + 32) of the segment; the source
      // of the first and whether all 32 are that source's (looked up while the
      // accumulator fills)
      int src = 0, src_end = 0, drow = 0, lr0 = 0;
      const int* sb = nullptr;
      const int* rr = nullptr;
      if (MODE == 1) {
        sb = args.lay->src_begin + c.j * (kMaxWorld + 1);
        rr = args.lay->ret_row + c.j * kMaxWorld;
        lr0 = c.row0 - S->base[c.j] + (int)cta * 128 + q * 32;
        while (src + 1 < args.world && __ldg(sb + src + 1) <= lr0) ++src;
        src_end = __ldg(sb + src + 1);
        drow = __ldg(rr + src) + (lr0 - __ldg(sb + src));
      }
      // one lane waits, the warp follows its verdict: the TMEM loads below are
      // warp-collective, so the warp must never split on a timeout
      int ok = 1;
      if (lane == 0) ok = mbar_wait(&S->tfull[b], aph, S, args.err);
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) break;
      fence_after();
      const uint32_t tbase = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(b * BN);
      // drain this warp's TMEM columns into registers, hand the accumulator
      // back to the MMA warp, then store
      uint32_t packed[2][32];
      if (MODE == 0) {
        // act columns [h*64, h*64+64) of this tile: gate at TMEM columns
        // h*64.., up at 128 + h*64..
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          uint32_t g[32], u[32];
          const int col = h * 64 + half * 32;
          tmem_ld32(tbase + col, g);
          tmem_ld32(tbase + 128 + col, u);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 16; ++i)
            packed[0][half * 16 + i] =
                pack_bf16x2(swiglu_bf16(__uint_as_float(g[2 * i]), __uint_as_float(u[2 * i])),
                            swiglu_bf16(__uint_as_float(g[2 * i + 1]), __uint_as_float(u[2 * i + 1])));
        }
      } else {
        // output columns [h*128, h*128+128) of this tile, 64 at a time
#pragma unroll
        for (int c64 = 0; c64 < 2; ++c64) {
          uint32_t y0[32], y1[32];
          const int col = h * 128 + c64 * 64;
          tmem_ld32(tbase + col, y0);
          tmem_ld32(tbase + col + 32, y1);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            packed[c64][i] = pack_bf16x2(__uint_as_float(y0[2 * i]), __uint_as_float(y0[2 * i + 1]));
            packed[c64][16 + i] =
                pack_bf16x2(__uint_as_float(y1[2 * i]), __uint_as_float(y1[2 * i + 1]));
          }
        }
      }
      fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(tempty_leader[b]);
      if (MODE == 0) {
        bf16* row = valid ? args.act + grow * args.act_ld + c.nb * 128 + h * 64 : nullptr;
        warp_store_rows(stage, packed[0], row, lane);
      } else {
        const int col0 = c.nb * BN + h * 128;
        if (lane == 0)  // the staging area's previous tile stores have read it
          asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
        __syncwarp();
        if (lr0 + 32 <= src_end) {
          // one source's contiguous rows: two 32 x 64 tile stores into its
          // return buffer (a peer's over NVLink), issued by one lane
#pragma unroll
          for (int c64 = 0; c64 < 2; ++c64) {
            if (c64) {
              if (lane == 0) asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
              __syncwarp();
            }
            uint8_t* srow = stage + lane * 128;
#pragma unroll
            for (int i = 0; i < 8; ++i)
              *reinterpret_cast<uint4*>(srow + ((i ^ (lane & 7)) << 4)) =
                  make_uint4(packed[c64][4 * i], packed[c64][4 * i + 1], packed[c64][4 * i + 2],
                             packed[c64][4 * i + 3]);
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            __syncwarp();
            if (lane == 0) {
              tma_store_2d(&rmaps.m[src], stage, col0 + c64 * 64, drow);
              asm volatile("cp.async.bulk.commit_group;" ::: "memory");
            }
          }
        } else {
          // the chunk crosses a source boundary or the segment's end: row by row
          const int lr = lr0 + lane;
          bf16* row = nullptr;
          if (lr < S->rows[c.j]) {
            int s2 = src;
            while (s2 + 1 < args.world && __ldg(sb + s2 + 1) <= lr) ++s2;
            row = static_cast<bf16*>(args.peers.ret[s2]) +
                  (int64_t)(__ldg(rr + s2) + lr - __ldg(sb + s2)) * args.H + col0;
          }
          warp_store_rows(stage, packed[0], row, lane);
          warp_store_rows(stage, packed[1], row ? row + 64 : nullptr, lane);
        }
      }
    }
    if (MODE == 1 && lane == 0) {
      // every tile store has written its rows before the completion signal
      asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
      asm volatile("fence.proxy.async.global;" ::: "memory");
    }
  }

  fence_before();
  __syncthreads();
  if (PAIR) cluster_sync();  // the pair's MMAs and remote arrivals are over before TMEM is freed
  fence_after();
  if (wp == 1) {
    if (PAIR)
      asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base),
                   "r"(TMEM_COLS)
                   : "memory");
    else
      asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base),
                   "r"(TMEM_COLS)
                   : "memory");
  }
  if (MODE == 1) grid_done_signal_ffn(args.done_ctr, args.peers, args.world, args.rank, args.seq);
  tl_end(args.tl, (MODE == 0 ? kTlGemm1 : kTlGemm2) + 1);
}

PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

int make_tmap(CUtensorMap* m, const void* base, uint64_t inner, uint64_t outer,
              uint32_t box_outer) {
  return encode_bf16_2d(m, base, inner, outer, BK, box_outer);
}

}  // namespace ffn
}  // namespace

// bf16 2D tensor map (rows of `inner` elements, `outer` rows), box
// box_inner x box_outer, 128-byte swizzle
int encode_bf16_2d(CUtensorMap* m, const void* base, uint64_t inner, uint64_t outer,
                   uint32_t box_inner, uint32_t box_outer) {
  if (int rc = tc_init()) return rc;
  const cuuint64_t dims[2] = {inner, outer};
  const cuuint64_t strides[1] = {inner * 2};
  const cuuint32_t box[2] = {box_inner, box_outer};
  const cuuint32_t es[2] = {1, 1};
  const CUresult r = ffn::g_encode(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base),
                                  dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : -100 - (int)r;
}

bool tc_shape_ok(int hidden, int inter) {
  return hidden % ffn::BN == 0 && inter % 128 == 0;
}

int tc_init() {
  if (ffn::g_encode) return 0;
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult q;
  const cudaError_t e =
      cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
  if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !fn) return -1;
  if (cudaFuncSetAttribute(ffn::k_ffn_tc<0, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           ffn::smem_bytes<false>()) != cudaSuccess ||
      cudaFuncSetAttribute(ffn::k_ffn_tc<1, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           ffn::smem_bytes<false>()) != cudaSuccess ||
      cudaFuncSetAttribute(ffn::k_ffn_tc<0, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           ffn::smem_bytes<true>()) != cudaSuccess ||
      cudaFuncSetAttribute(ffn::k_ffn_tc<1, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           ffn::smem_bytes<true>()) != cudaSuccess ||
      cudaFuncSetAttribute(ffn::k_ffn_tc<1, true, true>,
                           cudaFuncAttributeMaxDynamicSharedMemorySize,
                           ffn::smem_bytes<true, true>()) != cudaSuccess)
    return -2;
  ffn::g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  return 0;
}

int launch_ffn(const FfnArgs& a, cudaStream_t st) {
  const int H = a.hidden, I = a.inter;
  const bool use_tc = a.dtype == kBF16 && !a.force_simt && tc_shape_ok(H, I);
  if (use_tc) {
    int rc = tc_init();
    if (rc) return rc;
    CUtensorMap tmA1, tmB1, tmA2, tmB2;
    const uint64_t nl = (uint64_t)(a.n_local_weights > 0 ? a.n_local_weights : 1);
    if ((rc = ffn::make_tmap(&tmA1, a.recv_x, H, a.cap_rows, 128))) return rc;
    if ((rc = ffn::make_tmap(&tmA2, a.act, I, a.cap_rows, 128))) return rc;
    if ((rc = ffn::make_tmap(&tmB1, a.w_in, H, nl * 2 * I, 128))) return rc;
    if ((rc = ffn::make_tmap(&tmB2, a.w_out, I, nl * H, 128))) return rc;
    ffn::TcArgs g1{};
    g1.lay = a.layout;
    g1.K = H;
    g1.ntiles_n = I / 128;
    g1.b_rows_per_expert = 2 * I;
    g1.b_step = 128;
    g1.b_second = I;
    g1.act = static_cast<bf16*>(a.act);
    g1.act_ld = I;
    g1.err = a.err;
    g1.tl = a.tl;
    g1.prefetch = a.prefetch;
    const bool pair = !a.tc_single_cta && a.num_sms >= 2;
    // CTA pairs: 2-CTA clusters over an even grid; single CTAs: one per SM
    // GEMM2's tile stores: every rank's return buffer (ranks past world: unused)
    ffn::RetMaps rmaps;
    std::memset(&rmaps, 0, sizeof(rmaps));
    for (int r = 0; r < a.world; ++r)
      if ((rc = ffn::make_tmap(&rmaps.m[r], a.peers.ret[r], H, (uint64_t)a.ret_rows, 32)))
        return rc;
    auto launch = [&](auto kernel, bool as_pair, const CUtensorMap& ta, const CUtensorMap& tb,
                      const ffn::TcArgs& g, int smem) -> cudaError_t {
      cudaLaunchConfig_t cfg{};
      cfg.gridDim = dim3((unsigned)(as_pair ? (a.num_sms & ~1) : a.num_sms));
      cfg.blockDim = dim3(ffn::THREADS);
      cfg.dynamicSmemBytes = smem;
      cfg.stream = st;
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeClusterDimension;
      attr[0].val.clusterDim.x = as_pair ? 2 : 1;
      attr[0].val.clusterDim.y = 1;
      attr[0].val.clusterDim.z = 1;
      cfg.attrs = attr;
      cfg.numAttrs = as_pair ? 1 : 0;
      return cudaLaunchKernelEx(&cfg, kernel, ta, tb, rmaps, g);
    };
    cudaError_t e = pair ? launch(ffn::k_ffn_tc<0, true>, true, tmA1, tmB1, g1,
                                  ffn::smem_bytes<true>())
                         : launch(ffn::k_ffn_tc<0, false>, false, tmA1, tmB1, g1,
                                  ffn::smem_bytes<false>());
    if (e != cudaSuccess) return (int)e;
    ffn::TcArgs g2{};
    g2.lay = a.layout;
    g2.K = I;
    g2.ntiles_n = H / ffn::BN;
    g2.b_rows_per_expert = H;
    g2.b_step = ffn::BN;
    g2.b_second = 128;
    g2.peers = a.peers;
    g2.H = H;
    g2.world = a.world;
    g2.rank = a.rank;
    g2.done_ctr = a.done_ctr;
    g2.seq = a.seq;
    g2.err = a.err;
    g2.tl = a.tl;
    g2.prefetch = a.prefetch;
    // A-stationary GEMM2 when a row tile's A (K = I columns) fits the resident slots
    const bool ast = pair && a.ast && I / ffn::BK <= ffn::AST_SLOTS;
    if (ast)
      e = launch(ffn::k_ffn_tc<1, true, true>, true, tmA2, tmB2, g2,
                 ffn::smem_bytes<true, true>());
    else
      e = pair ? launch(ffn::k_ffn_tc<1, true>, true, tmA2, tmB2, g2, ffn::smem_bytes<true>())
               : launch(ffn::k_ffn_tc<1, false>, false, tmA2, tmB2, g2, ffn::smem_bytes<false>());
    if (e != cudaSuccess) return (int)e;
    return (int)cudaGetLastError();
  }
  if (H % kSimtBN != 0 || I % 32 != 0) return -3;
  const unsigned grid = (unsigned)a.num_sms * 4;
  if (a.dtype == kBF16) {
    k_ffn_simt<bf16, 0><<<grid, 256, 0, st>>>(
        static_cast<const bf16*>(a.recv_x), H, static_cast<const bf16*>(a.w_in), H, 2 * I, I,
        I / 32, a.layout, static_cast<bf16*>(a.act), I, a.peers, H, a.world, a.rank,
        nullptr, a.seq, a.tl);
    k_ffn_simt<bf16, 1><<<grid, 256, 0, st>>>(
        static_cast<const bf16*>(a.act), I, static_cast<const bf16*>(a.w_out), I, H, 0,
        H / kSimtBN, a.layout, nullptr, 0, a.peers, H, a.world, a.rank, a.done_ctr,
        a.seq, a.tl);
  } else {
    k_ffn_simt<float, 0><<<grid, 256, 0, st>>>(
        static_cast<const float*>(a.recv_x), H, static_cast<const float*>(a.w_in), H, 2 * I, I,
        I / 32, a.layout, static_cast<float*>(a.act), I, a.peers, H, a.world, a.rank,
        nullptr, a.seq, a.tl);
    k_ffn_simt<float, 1><<<grid, 256, 0, st>>>(
        static_cast<const float*>(a.act), I, static_cast<const float*>(a.w_out), I, H, 0,
        H / kSimtBN, a.layout, nullptr, 0, a.peers, H, a.world, a.rank,
        a.done_ctr, a.seq, a.tl);
  }
  return (int)cudaGetLastError();
}

}  // namespace mep
