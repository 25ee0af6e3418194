// Expert FFN over the expert-grouped receive buffer (run_experts,
// miniep/modeling.py:83-104):
//     h   = x_e @ w_in[e]^T            (rounded to the model dtype)
//     act = silu(h[:, :I]) * h[:, I:]  (each op rounded to the model dtype)
//     y   = act @ w_out[e]^T           (rounded), stored straight back to the
//                                      source rank's (token, slot) landing row.
//
// Two implementations share the tile schedule (Layout: expert segments padded
// to 128 rows, tile t -> (segment, 128-row block, N block)):
//   * tcgen05 (bf16): persistent, warp-specialised kernel. Warp 0 issues TMA
//     loads (128B-swizzled K-major tiles) into a 4-stage shared-memory ring,
//     warp 1 issues tcgen05.mma (M=128, N=256, K=16) into a double-buffered
//     TMEM accumulator (2 x 256 columns), warps 2-5 drain TMEM with
//     tcgen05.ld and run the epilogue (SwiGLU, or the store to the source
//     rank's landing buffer over NVLink) while the next tile accumulates.
//     GEMM1 puts the gate rows [n, n+128) and the up rows [I+n, I+n+128) of
//     w_in side by side in one 256-row B tile, so one MMA chain produces both
//     halves of the SwiGLU for the same rows.
//   * CUDA cores (fp32, and bf16 when asked): 64x64 register-tiled FMA kernel.
#include <cstdint>
#include <cuda.h>
#include <cudaTypedefs.h>
#include "mep_device.cuh"

namespace mep {
namespace {

using bf16 = __nv_bfloat16;

__device__ __forceinline__ void grid_done_signal_ffn(unsigned int* done_ctr, const PeerPtrs& peers,
                                                     int world, int rank, uint32_t seq) {
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned prev = atomicAdd(done_ctr, 1u);
    if (prev == gridDim.x - 1) {
      __threadfence_system();
      for (int d = 0; d < world; ++d) st_release_sys(peers.flags[d] + 2 * world + rank, seq);
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
                                                  const int32_t* __restrict__ meta, PeerPtrs peers,
                                                  int H, int world, int rank,
                                                  unsigned int* done_ctr, uint32_t seq) {
  __shared__ float As[kSimtBK][kSimtBM + 4];
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
      for (int i = tid; i < kSimtBM * kSimtBN; i += 256) {
        const int r = i / kSimtBN, cc = i % kSimtBN;
        if (r < c.rows) {
          const int32_t mt = meta[c.row0 + r];
          T* dst = static_cast<T*>(peers.yk[mt >> 24]) + (int64_t)(mt & 0xffffff) * H;
          dst[c.nb * kSimtBN + cc] = Elt<T>::from_f(Cs[r][cc]);
        }
      }
    }
    __syncthreads();
  }
  if (MODE == 1) grid_done_signal_ffn(done_ctr, peers, world, rank, seq);
}

// =================================================================== tcgen05
namespace tc {
constexpr int BM = 128, BN = 256, BK = 64, STAGES = 4;
constexpr int A_STAGE = BM * BK * 2;            // 16 KiB
constexpr int B_STAGE = BN * BK * 2;            // 32 KiB
constexpr int DATA = STAGES * (A_STAGE + B_STAGE);
constexpr int THREADS = 192;                    // warp0 TMA, warp1 MMA, warps 2-5 epilogue
constexpr int TMEM_COLS = 512;                  // two 256-column fp32 accumulators
constexpr unsigned long long kWaitNs = 2000000000ull;  // bounded mbarrier waits (2 s)
// kind::f16 instruction descriptor: D f32, A/B bf16, both K-major, N=256, M=128
constexpr uint32_t IDESC = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) |
                           ((uint32_t)(BM >> 4) << 24);

struct Smem {
  uint64_t full[STAGES], empty[STAGES], tfull[2], tempty[2];
  uint32_t tmem_base;
  int abort;
  int n_local, total;
  int prefix[kMaxExperts + 1], base[kMaxExperts], rows[kMaxExperts];
};
// epilogue staging: each epilogue warp owns 32 rows x 128 B (+16 B pad against bank conflicts)
constexpr int STAGE_ROW_BYTES = 144;
constexpr int STAGE_WARP_BYTES = 32 * STAGE_ROW_BYTES;
constexpr int SMEM_OFF_STAGE = DATA + (((int)sizeof(Smem) + 127) / 128) * 128;
constexpr int SMEM_BYTES = SMEM_OFF_STAGE + 4 * STAGE_WARP_BYTES + 1024;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void mbar_init(uint64_t* b, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(b)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* b, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(b)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* b) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(b)) : "memory");
}
__device__ __forceinline__ bool mbar_try(uint64_t* b, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(b)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait: false (and the CTA abort flag + device error set) on timeout
// or when another role of this CTA already gave up.
__device__ __forceinline__ bool mbar_wait(uint64_t* b, uint32_t parity, Smem* S, int* err) {
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
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* tm, int x, int y,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(tm)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  uint64_t d = (uint64_t)((saddr & 0x3FFFFu) >> 4);
  d |= (uint64_t)1 << 16;             // leading byte offset (unused for swizzled K-major)
  d |= (uint64_t)(1024 >> 4) << 32;   // stride byte offset: 8 rows x 128 B
  d |= (uint64_t)1 << 46;             // descriptor version for tcgen05
  d |= (uint64_t)2 << 61;             // 128-byte swizzle
  return d;
}
__device__ __forceinline__ void mma_f16(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc,
                                        uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a), "l"(b), "r"(idesc), "r"(accumulate));
}
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ uint32_t pack_bf16x2(float a, float b) {
  const __nv_bfloat162 p = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&p);
}

// Store this warp's 32 rows x 64 bf16 columns (128 B per row): lane l holds row
// l's 32 packed words in v and that row's destination in dst (nullptr = skip).
// The rows go through the warp's shared-memory slice so that every store
// instruction writes four whole 128-byte row segments (coalesced for HBM and
// for NVLink when the destination is a peer's buffer).
__device__ __forceinline__ void warp_store_rows(uint8_t* stage, const uint32_t (&v)[32],
                                                void* dst, int lane) {
  uint4* srow = reinterpret_cast<uint4*>(stage + lane * STAGE_ROW_BYTES);
#pragma unroll
  for (int i = 0; i < 8; ++i) srow[i] = make_uint4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
  __syncwarp();
  const unsigned long long mine = reinterpret_cast<unsigned long long>(dst);
#pragma unroll
  for (int it = 0; it < 8; ++it) {
    const int r = it * 4 + (lane >> 3), seg = lane & 7;
    const unsigned long long d = __shfl_sync(0xffffffffu, mine, r);
    const uint4 val = *reinterpret_cast<const uint4*>(stage + r * STAGE_ROW_BYTES + seg * 16);
    if (d) reinterpret_cast<uint4*>(d)[seg] = val;
  }
  __syncwarp();
}

struct TcArgs {
  const Layout* lay;
  int K;                   // reduction length
  int ntiles_n;            // N blocks per 128-row tile
  int b_rows_per_expert;   // rows of B per local expert (2I or H)
  int b_step;              // B rows advanced per N block (128 for GEMM1, 256 for GEMM2)
  int b_second;            // offset of the second 128-row half of the B tile
  bf16* act;               // MODE 0 output
  int act_ld;
  const int32_t* meta;     // MODE 1: (src << 24) | entry per receive row
  PeerPtrs peers;
  int H, world, rank;
  unsigned int* done_ctr;
  uint32_t seq;
  int* err;
};

// MODE 0: GEMM1 + SwiGLU -> act. MODE 1: GEMM2 -> source landing rows.
template <int MODE>
__global__ void __launch_bounds__(THREADS, 1) k_ffn_tc(const __grid_constant__ CUtensorMap tmA,
                                                       const __grid_constant__ CUtensorMap tmB,
                                                       const TcArgs args) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * A_STAGE;
  Smem* S = reinterpret_cast<Smem*>(smem + DATA);
  const int wp = warp_id(), lane = lane_id();

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&S->full[s], 1);
      mbar_init(&S->empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&S->tfull[b], 1);
      mbar_init(&S->tempty[b], 4);
    }
    S->abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (wp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(&S->tmem_base)),
                 "r"(TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  {
    const Layout* lay = args.lay;
    const int nl = lay->n_local;
    if (threadIdx.x == 0) {
      S->n_local = nl;
      S->total = lay->total_mtiles * args.ntiles_n;
    }
    for (int i = threadIdx.x; i <= nl; i += blockDim.x) S->prefix[i] = lay->tile_prefix[i];
    for (int i = threadIdx.x; i < nl; i += blockDim.x) {
      S->base[i] = lay->seg_base[i];
      S->rows[i] = lay->seg_rows[i];
    }
  }
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem_base = S->tmem_base;
  const int total = S->total;
  const int kblocks = args.K / BK;

  if (wp == 0) {
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0;
      for (int t = blockIdx.x; t < total; t += gridDim.x) {
        const TileCoord c =
            decode_tile(t, args.ntiles_n, 1, BM, kRowAlign, S->n_local, S->prefix, S->base, S->rows);
        const int brow0 = c.j * args.b_rows_per_expert + c.nb * args.b_step;
        const int brow1 = brow0 + args.b_second;
        bool ok = true;
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(&S->empty[s], ph ^ 1u, S, args.err)) {
            ok = false;
            break;
          }
          mbar_expect_tx(&S->full[s], A_STAGE + B_STAGE);
          tma_load_2d(sA + s * A_STAGE, &tmA, kb * BK, c.row0, &S->full[s]);
          tma_load_2d(sB + s * B_STAGE, &tmB, kb * BK, brow0, &S->full[s]);
          tma_load_2d(sB + s * B_STAGE + B_STAGE / 2, &tmB, kb * BK, brow1, &S->full[s]);
          if (++s == STAGES) {
            s = 0;
            ph ^= 1u;
          }
        }
        if (!ok) break;
      }
    }
  } else if (wp == 1) {
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0;
      int it = 0;
      for (int t = blockIdx.x; t < total; t += gridDim.x, ++it) {
        const int b = it & 1;
        const uint32_t aph = (uint32_t)(it >> 1) & 1u;
        if (!mbar_wait(&S->tempty[b], aph ^ 1u, S, args.err)) break;
        fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(b * BN);
        bool ok = true;
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(&S->full[s], ph, S, args.err)) {
            ok = false;
            break;
          }
          fence_after();
          const uint32_t a0 = smem_u32(sA + s * A_STAGE);
          const uint32_t b0 = smem_u32(sB + s * B_STAGE);
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk)
            mma_f16(d_tmem, sw128_desc(a0 + kk * 32), sw128_desc(b0 + kk * 32), IDESC,
                    (kb | kk) != 0);
          mma_commit(&S->empty[s]);
          if (++s == STAGES) {
            s = 0;
            ph ^= 1u;
          }
        }
        if (!ok) break;
        mma_commit(&S->tfull[b]);
      }
    }
  } else {
    // epilogue: warp w reads TMEM lanes [32*(w%4), 32*(w%4)+32)
    const int q = wp & 3;
    const int m = q * 32 + lane;
    int it = 0;
    for (int t = blockIdx.x; t < total; t += gridDim.x, ++it) {
      const int b = it & 1;
      const uint32_t aph = (uint32_t)(it >> 1) & 1u;
      // one lane waits, the warp follows its verdict: the TMEM loads below are
      // warp-collective, so the warp must never split on a timeout
      int ok = 1;
      if (lane == 0) ok = mbar_wait(&S->tfull[b], aph, S, args.err);
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) break;
      fence_after();
      const TileCoord c =
          decode_tile(t, args.ntiles_n, 1, BM, kRowAlign, S->n_local, S->prefix, S->base, S->rows);
      const bool valid = m < c.rows;
      const uint32_t tbase = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(b * BN);
      uint8_t* stage = smem + SMEM_OFF_STAGE + q * STAGE_WARP_BYTES;
      if (MODE == 0) {
        bf16* row = valid ? args.act + (int64_t)(c.row0 + m) * args.act_ld + c.nb * 128 : nullptr;
#pragma unroll 1
        for (int c64 = 0; c64 < 2; ++c64) {
          uint32_t packed[32];
#pragma unroll
          for (int half = 0; half < 2; ++half) {
            uint32_t g[32], u[32];
            const int col = c64 * 64 + half * 32;
            tmem_ld32(tbase + col, g);
            tmem_ld32(tbase + 128 + col, u);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              const float a0 =
                  silu_mul(__uint_as_float(g[2 * i]), __uint_as_float(u[2 * i]), true);
              const float a1 =
                  silu_mul(__uint_as_float(g[2 * i + 1]), __uint_as_float(u[2 * i + 1]), true);
              packed[half * 16 + i] = pack_bf16x2(a0, a1);
            }
          }
          warp_store_rows(stage, packed, row ? row + c64 * 64 : nullptr, lane);
        }
      } else {
        bf16* row = nullptr;
        if (valid) {
          const int32_t mt = args.meta[c.row0 + m];
          row = static_cast<bf16*>(args.peers.yk[mt >> 24]) + (int64_t)(mt & 0xffffff) * args.H +
                c.nb * BN;
        }
#pragma unroll 1
        for (int c64 = 0; c64 < BN / 64; ++c64) {
          uint32_t y0[32], y1[32], packed[32];
          tmem_ld32(tbase + c64 * 64, y0);
          tmem_ld32(tbase + c64 * 64 + 32, y1);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            packed[i] = pack_bf16x2(__uint_as_float(y0[2 * i]), __uint_as_float(y0[2 * i + 1]));
            packed[16 + i] =
                pack_bf16x2(__uint_as_float(y1[2 * i]), __uint_as_float(y1[2 * i + 1]));
          }
          warp_store_rows(stage, packed, row ? row + c64 * 64 : nullptr, lane);
        }
      }
      fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&S->tempty[b]);
    }
  }

  fence_before();
  __syncthreads();
  fence_after();
  if (wp == 1)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base),
                 "r"(TMEM_COLS)
                 : "memory");
  if (MODE == 1) grid_done_signal_ffn(args.done_ctr, args.peers, args.world, args.rank, args.seq);
}

// ---------------------------------------------------------------- CTA pairs
// The same FFN with a pair of CTAs (a 2-CTA cluster) per 256x256 tile: the
// leader CTA issues tcgen05.mma.cta_group::2 (M=256, N=256, K=16); each CTA
// holds its own 128 rows of A and 128 of the 256 B rows in its shared memory
// and its own 128 x 256 fp32 accumulator rows in its TMEM. Per k-block a CTA
// loads 32 KB instead of 48 KB for the same tensor work, and six stages fit.
// GEMM1's B split is natural: the leader loads the 128 gate rows, the other
// CTA the 128 up rows. Both CTAs' TMA loads complete on the leader's "full"
// barrier; the leader's MMA completion is committed to both CTAs' "empty" and
// "accumulator full" barriers; both CTAs' epilogue warps arrive on the
// leader's "accumulator empty" barrier. Expert segments are padded to 128
// rows, so the second CTA of a pair tile may hold rows past the segment end:
// those rows are computed and not stored.
constexpr int P_STAGES = 6;
constexpr int P_STAGE = A_STAGE + A_STAGE;           // 16 KB of A + 16 KB of B per CTA
constexpr int P_DATA = P_STAGES * P_STAGE;
constexpr uint32_t P_IDESC = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) |
                             ((uint32_t)(256 >> 4) << 24);

struct PSmem {
  uint64_t full[P_STAGES], empty[P_STAGES], tfull[2], tempty[2];
  uint32_t tmem_base;
  int abort;
  int n_local, total;
  int prefix[kMaxExperts + 1], base[kMaxExperts], rows[kMaxExperts];
};
constexpr int P_OFF_STAGE = P_DATA + (((int)sizeof(PSmem) + 127) / 128) * 128;
constexpr int P_SMEM_BYTES = P_OFF_STAGE + 4 * STAGE_WARP_BYTES + 1024;

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// shared::cluster address of the same location in CTA `cta` of this cluster
__device__ __forceinline__ uint32_t map_to_cta(const void* p, uint32_t cta) {
  uint32_t out;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(out) : "r"(smem_u32(p)), "r"(cta));
  return out;
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// TMA load into this CTA's shared memory whose bytes complete on the pair
// leader's barrier (given as a shared::cluster address)
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* tm, int x, int y,
                                                 uint32_t leader_bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(tm)), "r"(x), "r"(y), "r"(leader_bar)
      : "memory");
}
__device__ __forceinline__ void mma_f16_pair(uint32_t d_tmem, uint64_t a, uint64_t b,
                                             uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a), "l"(b), "r"(idesc), "r"(accumulate));
}
// completion of this thread's prior pair MMAs arrives on the barrier at the
// same offset in both CTAs of the pair
__device__ __forceinline__ void mma_commit_pair(uint64_t* bar) {
  const uint16_t both = 0x3;
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64"
      " [%0], %1;" ::"r"(smem_u32(bar)),
      "h"(both)
      : "memory");
}
__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_bar) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_bar)
               : "memory");
}
__device__ __forceinline__ bool mbar_wait_p(uint64_t* b, uint32_t parity, PSmem* S, int* err) {
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

template <int MODE>
__global__ void __launch_bounds__(THREADS, 1) k_ffn_tc_pair(const __grid_constant__ CUtensorMap tmA,
                                                            const __grid_constant__ CUtensorMap tmB,
                                                            const TcArgs args) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  PSmem* S = reinterpret_cast<PSmem*>(smem + P_DATA);
  const int wp = warp_id(), lane = lane_id();
  const uint32_t cta = cluster_rank();
  const bool leader = cta == 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < P_STAGES; ++s) {
      mbar_init(&S->full[s], 1);
      mbar_init(&S->empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&S->tfull[b], 1);
      mbar_init(&S->tempty[b], 8);  // 4 epilogue warps x 2 CTAs (used in the leader)
    }
    S->abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (wp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(&S->tmem_base)),
                 "r"(TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  {
    const Layout* lay = args.lay;
    const int nl = lay->n_local;
    if (threadIdx.x == 0) {
      // 256-row pair tiles per local expert
      int tiles = 0;
      for (int j = 0; j < nl; ++j) {
        S->prefix[j] = tiles;
        tiles += (lay->seg_rows[j] + 255) / 256;
      }
      S->prefix[nl] = tiles;
      S->n_local = nl;
      S->total = lay->total_mtiles > 0 ? tiles * args.ntiles_n : 0;
    }
    for (int i = threadIdx.x; i < nl; i += blockDim.x) {
      S->base[i] = lay->seg_base[i];
      S->rows[i] = lay->seg_rows[i];
    }
  }
  fence_before();
  __syncthreads();
  cluster_sync();  // the peer's barriers exist before any remote arrive or TMA completion
  fence_after();
  const uint32_t tmem_base = S->tmem_base;
  const int total = S->total;
  const int kblocks = args.K / BK;
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;

  if (wp == 0) {
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0;
      for (int t = pair; t < total; t += npairs) {
        const TileCoord c =
            decode_tile(t, args.ntiles_n, 1, 256, 256, S->n_local, S->prefix, S->base, S->rows);
        const int arow = c.row0 + (int)cta * 128;
        const int brow = c.j * args.b_rows_per_expert + c.nb * args.b_step +
                         (cta ? args.b_second : 0);
        bool ok = true;
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait_p(&S->empty[s], ph ^ 1u, S, args.err)) {
            ok = false;
            break;
          }
          if (leader) mbar_expect_tx(&S->full[s], 2 * P_STAGE);
          const uint32_t lbar = map_to_cta(&S->full[s], 0);
          uint8_t* st = smem + s * P_STAGE;
          tma_load_2d_pair(st, &tmA, kb * BK, arow, lbar);
          tma_load_2d_pair(st + A_STAGE, &tmB, kb * BK, brow, lbar);
          if (++s == P_STAGES) {
            s = 0;
            ph ^= 1u;
          }
        }
        if (!ok) break;
      }
    }
  } else if (wp == 1) {
    if (leader && lane == 0) {
      int s = 0;
      uint32_t ph = 0;
      int it = 0;
      for (int t = pair; t < total; t += npairs, ++it) {
        const int b = it & 1;
        const uint32_t aph = (uint32_t)(it >> 1) & 1u;
        if (!mbar_wait_p(&S->tempty[b], aph ^ 1u, S, args.err)) break;
        fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(b * BN);
        bool ok = true;
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait_p(&S->full[s], ph, S, args.err)) {
            ok = false;
            break;
          }
          fence_after();
          const uint32_t a0 = smem_u32(smem + s * P_STAGE);
          const uint32_t b0 = a0 + A_STAGE;
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk)
            mma_f16_pair(d_tmem, sw128_desc(a0 + kk * 32), sw128_desc(b0 + kk * 32), P_IDESC,
                         (kb | kk) != 0);
          mma_commit_pair(&S->empty[s]);
          if (++s == P_STAGES) {
            s = 0;
            ph ^= 1u;
          }
        }
        if (!ok) break;
        mma_commit_pair(&S->tfull[b]);
      }
    }
  } else {
    const int q = wp & 3;
    const int m = q * 32 + lane;
    const uint32_t leader_tempty[2] = {map_to_cta(&S->tempty[0], 0), map_to_cta(&S->tempty[1], 0)};
    uint8_t* stage = smem + P_OFF_STAGE + q * STAGE_WARP_BYTES;
    int it = 0;
    for (int t = pair; t < total; t += npairs, ++it) {
      const int b = it & 1;
      const uint32_t aph = (uint32_t)(it >> 1) & 1u;
      int ok = 1;
      if (lane == 0) ok = mbar_wait_p(&S->tfull[b], aph, S, args.err);
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) break;
      fence_after();
      const TileCoord c =
          decode_tile(t, args.ntiles_n, 1, 256, 256, S->n_local, S->prefix, S->base, S->rows);
      const int r = (int)cta * 128 + m;  // row inside the 256-row pair tile
      const bool valid = r < c.rows;
      const int64_t grow = c.row0 + r;
      const uint32_t tbase = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(b * BN);
      if (MODE == 0) {
        bf16* row = valid ? args.act + grow * args.act_ld + c.nb * 128 : nullptr;
#pragma unroll 1
        for (int c64 = 0; c64 < 2; ++c64) {
          uint32_t packed[32];
#pragma unroll
          for (int half = 0; half < 2; ++half) {
            uint32_t g[32], u[32];
            const int col = c64 * 64 + half * 32;
            tmem_ld32(tbase + col, g);
            tmem_ld32(tbase + 128 + col, u);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              const float a0 =
                  silu_mul(__uint_as_float(g[2 * i]), __uint_as_float(u[2 * i]), true);
              const float a1 =
                  silu_mul(__uint_as_float(g[2 * i + 1]), __uint_as_float(u[2 * i + 1]), true);
              packed[half * 16 + i] = pack_bf16x2(a0, a1);
            }
          }
          warp_store_rows(stage, packed, row ? row + c64 * 64 : nullptr, lane);
        }
      } else {
        bf16* row = nullptr;
        if (valid) {
          const int32_t mt = args.meta[grow];
          row = static_cast<bf16*>(args.peers.yk[mt >> 24]) + (int64_t)(mt & 0xffffff) * args.H +
                c.nb * BN;
        }
#pragma unroll 1
        for (int c64 = 0; c64 < BN / 64; ++c64) {
          uint32_t y0[32], y1[32], packed[32];
          tmem_ld32(tbase + c64 * 64, y0);
          tmem_ld32(tbase + c64 * 64 + 32, y1);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            packed[i] = pack_bf16x2(__uint_as_float(y0[2 * i]), __uint_as_float(y0[2 * i + 1]));
            packed[16 + i] =
                pack_bf16x2(__uint_as_float(y1[2 * i]), __uint_as_float(y1[2 * i + 1]));
          }
          warp_store_rows(stage, packed, row ? row + c64 * 64 : nullptr, lane);
        }
      }
      fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_remote(leader_tempty[b]);
    }
  }

  fence_before();
  __syncthreads();
  cluster_sync();  // the pair's MMAs and remote arrivals are over before TMEM is freed
  fence_after();
  if (wp == 1)
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base),
                 "r"(TMEM_COLS)
                 : "memory");
  if (MODE == 1) grid_done_signal_ffn(args.done_ctr, args.peers, args.world, args.rank, args.seq);
}

PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

int make_tmap(CUtensorMap* m, const void* base, uint64_t inner, uint64_t outer,
              uint32_t box_outer) {
  const cuuint64_t dims[2] = {inner, outer};
  const cuuint64_t strides[1] = {inner * 2};
  const cuuint32_t box[2] = {BK, box_outer};
  const cuuint32_t es[2] = {1, 1};
  const CUresult r = g_encode(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims,
                              strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                              CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : -100 - (int)r;
}

}  // namespace tc
}  // namespace

bool tc_shape_ok(int hidden, int inter) {
  return hidden % tc::BN == 0 && inter % 128 == 0;
}

int tc_init() {
  if (tc::g_encode) return 0;
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult q;
  const cudaError_t e =
      cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
  if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !fn) return -1;
  if (cudaFuncSetAttribute(tc::k_ffn_tc<0>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           tc::SMEM_BYTES) != cudaSuccess)
    return -2;
  if (cudaFuncSetAttribute(tc::k_ffn_tc<1>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           tc::SMEM_BYTES) != cudaSuccess)
    return -2;
  if (cudaFuncSetAttribute(tc::k_ffn_tc_pair<0>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           tc::P_SMEM_BYTES) != cudaSuccess)
    return -2;
  if (cudaFuncSetAttribute(tc::k_ffn_tc_pair<1>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           tc::P_SMEM_BYTES) != cudaSuccess)
    return -2;
  tc::g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
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
    if ((rc = tc::make_tmap(&tmA1, a.recv_x, H, a.cap_rows, tc::BM))) return rc;
    if ((rc = tc::make_tmap(&tmA2, a.act, I, a.cap_rows, tc::BM))) return rc;
    if ((rc = tc::make_tmap(&tmB1, a.w_in, H, nl * 2 * I, 128))) return rc;
    if ((rc = tc::make_tmap(&tmB2, a.w_out, I, nl * H, 128))) return rc;
    tc::TcArgs g1{};
    g1.lay = a.layout;
    g1.K = H;
    g1.ntiles_n = I / 128;
    g1.b_rows_per_expert = 2 * I;
    g1.b_step = 128;
    g1.b_second = I;
    g1.act = static_cast<bf16*>(a.act);
    g1.act_ld = I;
    g1.err = a.err;
    const bool pair = !a.tc_single_cta && a.num_sms >= 2;
    const int pair_grid = a.num_sms & ~1;
    auto launch_pair = [&](auto kernel, const CUtensorMap& ta, const CUtensorMap& tb,
                           const tc::TcArgs& g) -> cudaError_t {
      cudaLaunchConfig_t cfg{};
      cfg.gridDim = dim3((unsigned)pair_grid);
      cfg.blockDim = dim3(tc::THREADS);
      cfg.dynamicSmemBytes = tc::P_SMEM_BYTES;
      cfg.stream = st;
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeClusterDimension;
      attr[0].val.clusterDim.x = 2;
      attr[0].val.clusterDim.y = 1;
      attr[0].val.clusterDim.z = 1;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      return cudaLaunchKernelEx(&cfg, kernel, ta, tb, g);
    };
    if (pair) {
      const cudaError_t e = launch_pair(tc::k_ffn_tc_pair<0>, tmA1, tmB1, g1);
      if (e != cudaSuccess) return (int)e;
    } else {
      tc::k_ffn_tc<0><<<a.num_sms, tc::THREADS, tc::SMEM_BYTES, st>>>(tmA1, tmB1, g1);
    }
    tc::TcArgs g2{};
    g2.lay = a.layout;
    g2.K = I;
    g2.ntiles_n = H / tc::BN;
    g2.b_rows_per_expert = H;
    g2.b_step = tc::BN;
    g2.b_second = 128;
    g2.meta = a.recv_meta;
    g2.peers = a.peers;
    g2.H = H;
    g2.world = a.world;
    g2.rank = a.rank;
    g2.done_ctr = a.done_ctr;
    g2.seq = a.seq;
    g2.err = a.err;
    if (pair) {
      const cudaError_t e = launch_pair(tc::k_ffn_tc_pair<1>, tmA2, tmB2, g2);
      if (e != cudaSuccess) return (int)e;
    } else {
      tc::k_ffn_tc<1><<<a.num_sms, tc::THREADS, tc::SMEM_BYTES, st>>>(tmA2, tmB2, g2);
    }
    return (int)cudaGetLastError();
  }
  if (H % kSimtBN != 0 || I % 32 != 0) return -3;
  const unsigned grid = (unsigned)a.num_sms * 4;
  if (a.dtype == kBF16) {
    k_ffn_simt<bf16, 0><<<grid, 256, 0, st>>>(
        static_cast<const bf16*>(a.recv_x), H, static_cast<const bf16*>(a.w_in), H, 2 * I, I,
        I / 32, a.layout, static_cast<bf16*>(a.act), I, nullptr, a.peers, H, a.world, a.rank,
        nullptr, a.seq);
    k_ffn_simt<bf16, 1><<<grid, 256, 0, st>>>(
        static_cast<const bf16*>(a.act), I, static_cast<const bf16*>(a.w_out), I, H, 0,
        H / kSimtBN, a.layout, nullptr, 0, a.recv_meta, a.peers, H, a.world, a.rank, a.done_ctr,
        a.seq);
  } else {
    k_ffn_simt<float, 0><<<grid, 256, 0, st>>>(
        static_cast<const float*>(a.recv_x), H, static_cast<const float*>(a.w_in), H, 2 * I, I,
        I / 32, a.layout, static_cast<float*>(a.act), I, nullptr, a.peers, H, a.world, a.rank,
        nullptr, a.seq);
    k_ffn_simt<float, 1><<<grid, 256, 0, st>>>(
        static_cast<const float*>(a.act), I, static_cast<const float*>(a.w_out), I, H, 0,
        H / kSimtBN, a.layout, nullptr, 0, a.recv_meta, a.peers, H, a.world, a.rank,
        a.done_ctr, a.seq);
  }
  return (int)cudaGetLastError();
}

}  // namespace mep
