// Router on the tcgen05 tensor cores, for large token counts (bf16, E = 32 or
// 64 experts): logits = x @ router^T (miniep/modeling.py:193) per tile of up
// to 128 tokens, one tcgen05.mma chain (M = 128 rows, N = E, K = 16 per
// instruction) over TMA-loaded, 128B-swizzled K-slices of x and of the
// router rows, accumulated in TMEM in fp32 (double-buffered, so the next
// tile accumulates while this one is selected). One epilogue thread per
// token then rounds the logits to bf16, adds the bias (rounded), selects the
// top-k with ties to the lower expert index and takes the softmax over them
// in fp32 (modeling.py:194-195): the values and operations of the CUDA-core
// router's selection, so both give the same indices and gates for the same
// logits.
//
// Persistent: one CTA per SM walks the tiles, sized so that every SM gets one
// (a tile of tpt < 128 tokens loads tpt rows; the MMA's other rows are
// dropped). Warp 0 issues the TMA loads
// into an 8-stage ring, warp 1 the MMAs, warps 2-5 (one per TMEM lane
// quadrant) drain the accumulator. Every mbarrier wait is bounded.
#include <cmath>
#include <cstdint>
#include <cuda_bf16.h>
#include "mep_device.cuh"
#include "mep_tc.cuh"

namespace mep {
namespace {
namespace rt {
using namespace ::mep::tc;
using bf16 = __nv_bfloat16;

constexpr int TILE = 128;  // tokens per tile (MMA M)
constexpr int BK = 64;     // K per stage: one 128-byte swizzle row of bf16
constexpr int STAGES = 8;
constexpr int EPI_WARPS = 4;
constexpr int THREADS = 64 + 32 * EPI_WARPS;
constexpr unsigned long long kWaitNs = 2000000000ull;

template <int E>
struct Cfg {
  static constexpr int A_BYTES = TILE * BK * 2;         // 16 KiB of x
  static constexpr int B_BYTES = E * BK * 2;            // 4 / 8 KiB of router rows
  static constexpr int STAGE = A_BYTES + B_BYTES;       // a multiple of 1024
  static constexpr int DATA = STAGES * STAGE;
  // kind::f16: D f32, A and B bf16, both K-major, N = E, M = 128
  static constexpr uint32_t IDESC = (1u << 4) | (1u << 7) | (1u << 10) |
                                    ((uint32_t)(E >> 3) << 17) | ((uint32_t)(TILE >> 4) << 24);
  static constexpr uint32_t TMEM_COLS = 2 * E;          // two accumulators: 64 or 128 columns
};

struct Smem {
  uint64_t full[STAGES], empty[STAGES], tfull[2], tempty[2];
  uint32_t tmem_base;
  int abort;
  float bias[64];
};
static_assert(sizeof(Smem) <= 1024, "router barriers");

template <int E>
constexpr int smem_bytes() {
  return Cfg<E>::DATA + 1024 + 1024;  // data | barriers | alignment slack
}

struct RouterArgs {
  int64_t n;
  int H, k;
  int tpt;  // tokens per tile (<= TILE): the grid covers every SM even when n < TILE * SMs
  const float* bias;
  int64_t* idx_out;
  bf16* gate_out;
  float* logits_out;
  int* err;
  uint64_t* tl;
};

__device__ __forceinline__ bool wait_bar(uint64_t* b, uint32_t parity, Smem* S, int* err) {
  if (mbar_wait_for(b, parity, kWaitNs, &S->abort)) return true;
  set_err(err, kErrPipeline);
  return false;
}

template <int E>
__global__ void __launch_bounds__(THREADS, 1) k_router_tc(const __grid_constant__ CUtensorMap tmX,
                                                          const __grid_constant__ CUtensorMap tmW,
                                                          const RouterArgs a) {
  using C = Cfg<E>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  Smem* S = reinterpret_cast<Smem*>(smem + C::DATA);
  const int wp = warp_id(), lane = lane_id();
  tl_begin(a.tl, kTlRouter);
  if (threadIdx.x == 32) {
    tma_prefetch_desc(&tmX);
    tma_prefetch_desc(&tmW);
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&S->full[s], 1);
      mbar_init(&S->empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&S->tfull[b], 1);
      mbar_init(&S->tempty[b], EPI_WARPS);
    }
    S->abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (wp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(&S->tmem_base)),
                 "r"(C::TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  for (int e = threadIdx.x; e < E; e += blockDim.x) S->bias[e] = a.bias ? a.bias[e] : 0.f;
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = S->tmem_base;
  const int ntiles = (int)((a.n + a.tpt - 1) / a.tpt);
  const int kblocks = a.H / BK;

  if (wp == 0) {
    // ------------------------------------------------------------ TMA loads
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x) {
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!wait_bar(&S->empty[s], ph ^ 1u, S, a.err)) {
            ok = false;
            break;
          }
          mbar_expect_tx(&S->full[s], (uint32_t)(a.tpt * BK * 2 + C::B_BYTES));
          uint8_t* st = smem + s * C::STAGE;
          tma_load_2d<false>(st, &tmX, kb * BK, t * a.tpt, smem_u32(&S->full[s]));
          tma_load_2d<false>(st + C::A_BYTES, &tmW, kb * BK, 0, smem_u32(&S->full[s]));
          if (++s == STAGES) {
            s = 0;
            ph ^= 1u;
          }
        }
      }
    }
  } else if (wp == 1) {
    // ------------------------------------------------------------ MMA issue
    if (lane == 0) {
      int s = 0, it = 0;
      uint32_t ph = 0;
      for (int t = blockIdx.x; t < ntiles; t += gridDim.x, ++it) {
        const int b = it & 1;
        const uint32_t aph = (uint32_t)(it >> 1) & 1u;
        if (!wait_bar(&S->tempty[b], aph ^ 1u, S, a.err)) break;
        fence_after();
        const uint32_t d = tmem + (uint32_t)(b * E);
        bool ok = true;
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!wait_bar(&S->full[s], ph, S, a.err)) {
            ok = false;
            break;
          }
          fence_after();
          const uint32_t a0 = smem_u32(smem + s * C::STAGE);
          const uint32_t b0 = a0 + C::A_BYTES;
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk)
            mma_f16<false>(d, sw128_desc(a0 + kk * 32), sw128_desc(b0 + kk * 32), C::IDESC,
                           (kb | kk) != 0);
          mma_commit<false>(&S->empty[s]);
          if (++s == STAGES) {
            s = 0;
            ph ^= 1u;
          }
        }
        if (!ok) break;
        mma_commit<false>(&S->tfull[b]);
      }
    }
  } else {
    // ------------------------------------------------------------ selection
    const int q = wp & 3;  // this warp's TMEM lane quadrant: tokens q*32 .. q*32+31 of a tile
    int it = 0;
    for (int t = blockIdx.x; t < ntiles; t += gridDim.x, ++it) {
      const int b = it & 1;
      const uint32_t aph = (uint32_t)(it >> 1) & 1u;
      int ok = 1;
      if (lane == 0) ok = wait_bar(&S->tfull[b], aph, S, a.err);
      ok = __shfl_sync(0xffffffffu, ok, 0);  // the TMEM loads are warp-collective
      if (!ok) break;
      fence_after();
      const uint32_t tb = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(b * E);
      uint32_t r0[32], r1[32];
      tmem_ld32(tb, r0);
      if (E == 64) tmem_ld32(tb + 32, r1);
      tmem_wait_ld();
      fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&S->tempty[b]);
      // accumulator rows at or past tpt come from shared memory the tile's
      // load did not write: they are computed and dropped
      const int row = q * 32 + lane;
      const int64_t tok = (int64_t)t * a.tpt + row;
      if (row >= a.tpt || tok >= a.n) continue;
      float v[E];
#pragma unroll
      for (int e = 0; e < E; ++e) {
        const float acc = __uint_as_float(e < 32 ? r0[e] : r1[e & 31]);
        float l = bf16_round(acc);  // logits in the model dtype
        if (a.bias) l = bf16_round(l + bf16_round(S->bias[e]));
        v[e] = l;
      }
      if (a.logits_out) {
        float4* lo = reinterpret_cast<float4*>(a.logits_out + tok * E);
#pragma unroll
        for (int e = 0; e < E; e += 4) lo[e / 4] = make_float4(v[e], v[e + 1], v[e + 2], v[e + 3]);
      }
      // top-k: larger value first, the lower expert index on ties. The
      // logits are bf16 values, so each becomes one 32-bit key: its bf16
      // bits mapped to an unsigned order (-0 taken as +0) above 0xFFFF - e.
      // Keys are distinct and compare exactly as (value, then lower index),
      // so each round is a max-tree over E keys (short dependency chains)
      // instead of a serial scan. The rounds stay rolled: each CTA runs this
      // code for a tile or two, so its instruction fetch is what costs.
      uint32_t key[E];
#pragma unroll
      for (int e = 0; e < E; ++e) {
        uint32_t b = __float_as_uint(v[e]) >> 16;
        if ((b & 0x7FFFu) == 0u) b = 0u;
        const uint32_t ord = (b & 0x8000u) ? (~b & 0xFFFFu) : (b | 0x8000u);
        key[e] = (ord << 16) | (0xFFFFu - (uint32_t)e);
      }
      float top0 = 0.f, ex_sum = 0.f;
      float ex[kMaxTopk];
#pragma unroll 1
      for (int i = 0; i < a.k; ++i) {
        uint32_t t[E];
#pragma unroll
        for (int e = 0; e < E; ++e) t[e] = key[e];
#pragma unroll
        for (int w = E / 2; w > 0; w >>= 1)
#pragma unroll
          for (int e = 0; e < w; ++e) t[e] = max(t[e], t[e + w]);
        const uint32_t top = t[0];
#pragma unroll
        for (int e = 0; e < E; ++e) key[e] = key[e] == top ? 0u : key[e];  // taken
        const uint32_t ord = top >> 16;
        const uint32_t b = (ord & 0x8000u) ? (ord & 0x7FFFu) : (~ord & 0xFFFFu);
        const float best = __uint_as_float(b << 16);
        if (i == 0) top0 = best;
        ex[i] = expf(best - top0);
        ex_sum += ex[i];
        a.idx_out[tok * a.k + i] = (int64_t)(0xFFFFu - (top & 0xFFFFu));
      }
      const float rs = 1.f / ex_sum;
#pragma unroll 1
      for (int i = 0; i < a.k; ++i) a.gate_out[tok * a.k + i] = __float2bfloat16_rn(ex[i] * rs);
    }
  }
  fence_before();
  __syncthreads();
  fence_after();
  if (wp == 1)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(C::TMEM_COLS)
                 : "memory");
  tl_end(a.tl, kTlRouter + 1);
}

template <int E>
int launch(int64_t n, int hidden, int topk, const void* x, const void* router_w,
           const float* bias, int64_t* idx_out, void* gate_out, float* logits_out, int num_sms,
           int* err, uint64_t* tl, cudaStream_t st) {
  static bool attr_set = false;
  if (!attr_set) {
    if (cudaFuncSetAttribute(k_router_tc<E>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             smem_bytes<E>()) != cudaSuccess)
      return -1;
    attr_set = true;
  }
  // tiles of tpt tokens (a multiple of 8, the swizzle atom's rows): enough
  // tiles for every SM, at most TILE tokens each
  int64_t tpt = (n + num_sms - 1) / num_sms;
  tpt = (tpt + 7) / 8 * 8;
  if (tpt > TILE) tpt = TILE;
  CUtensorMap tmX, tmW;
  if (encode_bf16_2d(&tmX, x, (uint64_t)hidden, (uint64_t)n, BK, (uint32_t)tpt)) return -1;
  if (encode_bf16_2d(&tmW, router_w, (uint64_t)hidden, (uint64_t)E, BK, E)) return -1;
  RouterArgs a{n, hidden, topk, (int)tpt, bias, idx_out, static_cast<bf16*>(gate_out),
               logits_out, err, tl};
  const int64_t ntiles = (n + tpt - 1) / tpt;
  const unsigned grid = (unsigned)(ntiles < num_sms ? ntiles : num_sms);
  k_router_tc<E><<<grid, THREADS, smem_bytes<E>(), st>>>(tmX, tmW, a);
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

}  // namespace rt
}  // namespace

// 0 when the tensor-core router ran, nonzero when the caller should use the
// CUDA-core kernels (shape not covered, or set-up failed)
int launch_router_tc(int64_t n, int hidden, int experts, int topk, const void* x,
                     const void* router_w, const float* bias, int64_t* idx_out, void* gate_out,
                     float* logits_out, int num_sms, int* err, uint64_t* tl, cudaStream_t st) {
  if (hidden % rt::BK != 0 || n < 1) return 1;
  if (((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(router_w)) & 15u) != 0)
    return 1;
  if (experts == 32)
    return rt::launch<32>(n, hidden, topk, x, router_w, bias, idx_out, gate_out, logits_out,
                          num_sms, err, tl, st);
  if (experts == 64)
    return rt::launch<64>(n, hidden, topk, x, router_w, bias, idx_out, gate_out, logits_out,
                          num_sms, err, tl, st);
  return 1;
}

}  // namespace mep
