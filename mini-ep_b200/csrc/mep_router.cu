// Router: logits = x @ router^T (fp32 accumulate, rounded to the model dtype),
// optional additive bias (rounded to the model dtype), top-k with ties broken
// towards the lower expert index, softmax over the k selected logits in fp32,
// gates rounded to the model dtype.
// Follows miniep/modeling.py:193-195 (Block.forward router lines).
#include <cstdint>
#include <cuda_bf16.h>
#include "mep_device.cuh"

namespace mep {
namespace {

using bf16 = __nv_bfloat16;

// Selection + softmax for one token whose model-dtype logits sit in v[0..E).
template <typename T>
__device__ __forceinline__ void select_topk(const float* v, int E, int k, int64_t tok,
                                            int64_t* idx_out, T* gate_out) {
  uint64_t used[2] = {0ull, 0ull};
  float top_v[kMaxTopk];
  int top_i[kMaxTopk];
  for (int i = 0; i < k; ++i) {
    float best = 0.f;
    int bi = -1;
    for (int e = 0; e < E; ++e) {
      if ((used[e >> 6] >> (e & 63)) & 1ull) continue;
      const float ve = v[e];
      if (bi < 0 || ve > best) {  // strict '>' keeps the lower index on ties
        best = ve;
        bi = e;
      }
    }
    used[bi >> 6] |= 1ull << (bi & 63);
    top_v[i] = best;
    top_i[i] = bi;
  }
  const float m = top_v[0];
  float ex[kMaxTopk];
  float s = 0.f;
  for (int i = 0; i < k; ++i) {
    ex[i] = expf(top_v[i] - m);
    s += ex[i];
  }
  const float r = 1.f / s;
  for (int i = 0; i < k; ++i) {
    idx_out[tok * k + i] = top_i[i];
    gate_out[tok * k + i] = Elt<T>::from_f(ex[i] * r);
  }
}

// Warp-parallel top-k for one token: lane l holds the model-dtype logits of
// experts l and l+32 (-inf past E). k rounds of a 5-step shuffle argmax
// (larger value first, lower index on ties, as the serial rule); lanes < k
// write the result. E <= 64.
template <typename T>
__device__ __forceinline__ void select_topk_warp(float v0, float v1, int k, int64_t tok,
                                                 int64_t* idx_out, T* gate_out) {
  const int lane = lane_id();
  float my_v = 0.f, top0 = 0.f;
  int my_i = 0;
  float ex_sum = 0.f;
  for (int i = 0; i < k; ++i) {
    // this lane's best remaining candidate
    float bv = v0;
    int bi = lane;
    if (v1 > bv) {
      bv = v1;
      bi = lane + 32;
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
      if (ov > bv || (ov == bv && oi < bi)) {
        bv = ov;
        bi = oi;
      }
    }
    if (bi == lane) v0 = -INFINITY;
    if (bi == lane + 32) v1 = -INFINITY;
    if (i == 0) top0 = bv;
    const float e = expf(bv - top0);
    ex_sum += e;
    if (lane == i) {
      my_v = e;
      my_i = bi;
    }
  }
  if (lane < k) {
    idx_out[tok * k + lane] = my_i;
    gate_out[tok * k + lane] = Elt<T>::from_f(my_v * (1.f / ex_sum));
  }
}

// E <= 32: lane l holds expert l's model-dtype logit (-inf past E). A 32-lane
// bitonic sort on (value descending, index ascending) -- the selection
// order of the rounds above, ties to the lower index -- leaves the i-th
// choice in lane i after 15 compare-exchange steps. The softmax then runs as
// above: exp(v_i - v_0) on lanes < k, summed in slot order, one reciprocal.
// Same values and summation order as select_topk_warp, so the same bits.
template <typename T>
__device__ __forceinline__ void select_topk_sort32(float v, int k, int64_t tok, int64_t* idx_out,
                                                   T* gate_out) {
  const int lane = lane_id();
  int i = lane;
#pragma unroll
  for (int size = 2; size <= 32; size <<= 1) {
#pragma unroll
    for (int j = size >> 1; j > 0; j >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, v, j);
      const int oi = __shfl_xor_sync(0xffffffffu, i, j);
      const bool other_better = ov > v || (ov == v && oi < i);
      const bool lower = (lane & j) == 0;
      const bool desc = (lane & size) == 0;  // this block ends best-first
      if (lower == desc ? other_better : !other_better) {
        v = ov;
        i = oi;
      }
    }
  }
  const float top0 = __shfl_sync(0xffffffffu, v, 0);
  const float e = lane < k ? expf(v - top0) : 0.f;
  float ex_sum = 0.f;
  for (int s = 0; s < k; ++s) ex_sum += __shfl_sync(0xffffffffu, e, s);
  if (lane < k) {
    idx_out[tok * k + lane] = i;
    gate_out[tok * k + lane] = Elt<T>::from_f(e * (1.f / ex_sum));
  }
}

template <typename T>
__device__ __forceinline__ float logit_to_model(float acc, const float* bias, int e) {
  float l = Elt<T>::round(acc);
  if (bias) l = Elt<T>::round(l + Elt<T>::round(bias[e]));
  return l;
}

__device__ __forceinline__ void mma_bf16_16816(float (&c)[4], uint32_t a0, uint32_t a1,
                                               uint32_t a2, uint32_t a3, uint32_t b0,
                                               uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// bf16 router on the warp-level tensor-core path (the router GEMM is
// (N x H) x (H x E) with E <= 64: far too narrow for a TMEM tile to pay, and
// the kernel is bound by reading x once from HBM). A CTA owns 16 tokens and
// all E = 8*NT experts; its 4 warps split H into quarters (when H is a
// multiple of 256) so that enough loads are in flight, and their partial
// logits are added in warp order (fixed, so the result is deterministic).
// Each warp walks its columns in 64-column blocks: every lane loads two
// 16-byte pieces per row and uses them for four k16 steps (the same column
// permutation is applied to x and to the router rows, which leaves every dot
// product unchanged).
template <int NT>
__global__ void __launch_bounds__(128) k_router_bf16_mma(
    const bf16* __restrict__ x, const bf16* __restrict__ w, const float* __restrict__ bias,
    int64_t n, int H, int E, int k, int64_t* __restrict__ idx_out, bf16* __restrict__ gate_out,
    float* __restrict__ logits_out, uint64_t* tl) {
  __shared__ float part[4][16][NT * 8 + 1];
  const int wp = warp_id(), lane = lane_id();
  tl_begin(tl, kTlRouter);
  const int g = lane >> 2, q = lane & 3;
  const int64_t tok0 = (int64_t)blockIdx.x * 16;
  const int ksplit = (H % 256 == 0) ? 4 : 1;
  const int kchunk = H / ksplit;
  const int64_t ra = min(tok0 + g, n - 1), rb = min(tok0 + g + 8, n - 1);
  const bf16* xa = x + ra * H + q * 16;
  const bf16* xb = x + rb * H + q * 16;
  float acc[NT][4];
#pragma unroll
  for (int t = 0; t < NT; ++t) acc[t][0] = acc[t][1] = acc[t][2] = acc[t][3] = 0.f;

  if (wp < ksplit) {
    const int kbeg = wp * kchunk, kend = kbeg + kchunk;
    for (int kb = kbeg; kb < kend; kb += 64) {
      const uint4 alo = __ldg(reinterpret_cast<const uint4*>(xa + kb));
      const uint4 ahi = __ldg(reinterpret_cast<const uint4*>(xa + kb + 8));
      const uint4 blo = __ldg(reinterpret_cast<const uint4*>(xb + kb));
      const uint4 bhi = __ldg(reinterpret_cast<const uint4*>(xb + kb + 8));
      const uint32_t ra_lo[4] = {alo.x, alo.y, alo.z, alo.w};  // row g, columns [0,8)
      const uint32_t ra_hi[4] = {ahi.x, ahi.y, ahi.z, ahi.w};  // row g, columns [8,16)
      const uint32_t rb_lo[4] = {blo.x, blo.y, blo.z, blo.w};  // row g+8
      const uint32_t rb_hi[4] = {bhi.x, bhi.y, bhi.z, bhi.w};
#pragma unroll
      for (int t = 0; t < NT; ++t) {
        const int ne = t * 8 + g;
        uint4 wlo = make_uint4(0, 0, 0, 0), whi = make_uint4(0, 0, 0, 0);
        if (ne < E) {
          const bf16* wr = w + (int64_t)ne * H + kb + q * 16;
          wlo = __ldg(reinterpret_cast<const uint4*>(wr));
          whi = __ldg(reinterpret_cast<const uint4*>(wr + 8));
        }
        const uint32_t w_lo[4] = {wlo.x, wlo.y, wlo.z, wlo.w};
        const uint32_t w_hi[4] = {whi.x, whi.y, whi.z, whi.w};
#pragma unroll
        for (int j = 0; j < 4; ++j)
          mma_bf16_16816(acc[t], ra_lo[j], rb_lo[j], ra_hi[j], rb_hi[j], w_lo[j], w_hi[j]);
      }
    }
  }
#pragma unroll
  for (int t = 0; t < NT; ++t) {
    part[wp][g][t * 8 + 2 * q] = acc[t][0];
    part[wp][g][t * 8 + 2 * q + 1] = acc[t][1];
    part[wp][g + 8][t * 8 + 2 * q] = acc[t][2];
    part[wp][g + 8][t * 8 + 2 * q + 1] = acc[t][3];
  }
  __syncthreads();
  // each warp selects for 4 of the 16 tokens, one expert per lane (two for E > 32)
  for (int r = wp * 4; r < wp * 4 + 4; ++r) {
    const int64_t tok = tok0 + r;
    if (tok >= n) break;
    float v[2];
#pragma unroll
    for (int h2 = 0; h2 < 2; ++h2) {
      const int e = lane + 32 * h2;
      if (e < E) {
        float sum = part[0][r][e];
        for (int w2 = 1; w2 < ksplit; ++w2) sum += part[w2][r][e];
        v[h2] = logit_to_model<bf16>(sum, bias, e);
        if (logits_out) logits_out[tok * E + e] = v[h2];
      } else {
        v[h2] = -INFINITY;
      }
    }
    if (NT <= 4)
      select_topk_sort32<bf16>(v[0], k, tok, idx_out, gate_out);
    else
      select_topk_warp<bf16>(v[0], v[1], k, tok, idx_out, gate_out);
  }
  tl_end(tl, kTlRouter + 1);
}

// CUDA-core router for fp32 (and any shape the tensor-core path does not take):
// one warp per token, lane e owns experts e, e+32, ...; plain fp32 FMA chains.
template <typename T>
__global__ void __launch_bounds__(128) k_router_simt(
    const T* __restrict__ x, const T* __restrict__ w, const float* __restrict__ bias, int64_t n,
    int H, int E, int k, int64_t* __restrict__ idx_out, T* __restrict__ gate_out,
    float* __restrict__ logits_out, uint64_t* tl) {
  __shared__ float sl[4][kMaxExperts];
  const int wp = warp_id(), lane = lane_id();
  const int64_t tok = (int64_t)blockIdx.x * 4 + wp;
  tl_begin(tl, kTlRouter);
  if (tok >= n) return;
  const T* xr = x + tok * H;
  for (int e = lane; e < E; e += 32) {
    const T* wr = w + (int64_t)e * H;
    float acc = 0.f;
    for (int h = 0; h < H; ++h) acc = fmaf(Elt<T>::to_f(xr[h]), Elt<T>::to_f(wr[h]), acc);
    sl[wp][e] = logit_to_model<T>(acc, bias, e);
  }
  __syncwarp();
  if (lane == 0) {
    float* v = sl[wp];
    if (logits_out)
      for (int e = 0; e < E; ++e) logits_out[tok * E + e] = v[e];
    select_topk<T>(v, E, k, tok, idx_out, gate_out);
  }
  tl_end(tl, kTlRouter + 1);
}

}  // namespace

void launch_router(int dtype, const void* x, const void* router_w, const float* bias, int64_t n,
                   int hidden, int experts, int topk, int64_t* idx_out, void* gate_out,
                   float* logits_out, int num_sms, int use_tc, int* err, uint64_t* tl,
                   cudaStream_t st) {
  if (n <= 0) return;
  // large batches: the tcgen05 router (TMA-fed, one CTA per SM); it covers
  // bf16 with 32 or 64 experts and rows on 16-byte boundaries
  if (dtype == kBF16 && use_tc && n >= kRouterTcMinTokens &&
      launch_router_tc(n, hidden, experts, topk, x, router_w, bias, idx_out, gate_out,
                       logits_out, num_sms, err, tl, st) == 0)
    return;
  // the warp-level tensor-core kernel reads x and the router rows in 16-byte
  // pieces; the CUDA-core kernel takes any layout
  const bool aligned16 = ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(router_w)) &
                          15u) == 0;
  if (dtype == kBF16 && hidden % 64 == 0 && experts % 8 == 0 && experts <= 64 && aligned16) {
    const unsigned grid = (unsigned)((n + 15) / 16);
    auto xb = static_cast<const bf16*>(x);
    auto wb = static_cast<const bf16*>(router_w);
    auto gb = static_cast<bf16*>(gate_out);
    switch (experts / 8) {
#define MEP_ROUTER_CASE(NT)                                                                   \
  case NT:                                                                                   \
    k_router_bf16_mma<NT><<<grid, 128, 0, st>>>(xb, wb, bias, n, hidden, experts, topk, idx_out, \
                                                gb, logits_out, tl);                         \
    return;
      MEP_ROUTER_CASE(1)
      MEP_ROUTER_CASE(2)
      MEP_ROUTER_CASE(3)
      MEP_ROUTER_CASE(4)
      MEP_ROUTER_CASE(5)
      MEP_ROUTER_CASE(6)
      MEP_ROUTER_CASE(7)
      MEP_ROUTER_CASE(8)
#undef MEP_ROUTER_CASE
    }
  }
  const unsigned grid = (unsigned)((n + 3) / 4);
  if (dtype == kBF16)
    k_router_simt<bf16><<<grid, 128, 0, st>>>(static_cast<const bf16*>(x),
                                              static_cast<const bf16*>(router_w), bias, n, hidden,
                                              experts, topk, idx_out, static_cast<bf16*>(gate_out),
                                              logits_out, tl);
  else
    k_router_simt<float><<<grid, 128, 0, st>>>(static_cast<const float*>(x),
                                               static_cast<const float*>(router_w), bias, n,
                                               hidden, experts, topk, idx_out,
                                               static_cast<float*>(gate_out), logits_out, tl);
}

}  // namespace mep
