// Post-attention RMSNorm of the MoE block: x = w * (h * rsqrt(mean(h^2) + eps))
// (miniep/modeling.py:51-52 and :192), in the model dtype with the reference's
// rounding points: each square rounded, the mean (fp32 sum) rounded, mean + eps
// rounded, 1/sqrt rounded, h * r rounded, w * (h * r) rounded. fp32 rounds
// nowhere. One warp per row; the row stays in registers (16-byte loads).
#include <cstdint>
#include <cuda_bf16.h>
#include "mep_device.cuh"

namespace mep {
namespace {

template <typename T>
struct Pack16 {
  static constexpr int N = 16 / sizeof(T);
};

__device__ __forceinline__ float bf16_bits_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16_bits_hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

// VPL 16-byte vectors per lane; H = 32 * VPL * (16 / sizeof(T))
template <typename T, int VPL>
__global__ void __launch_bounds__(256) k_rmsnorm(int64_t n, int H, const T* __restrict__ h,
                                                 const T* __restrict__ w, float eps,
                                                 T* __restrict__ x, uint64_t* tl) {
  constexpr int V = Pack16<T>::N;
  const int lane = lane_id();
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + warp_id();
  tl_begin(tl, kTlNorm);
  if (row >= n) return;
  const uint4* hr = reinterpret_cast<const uint4*>(h + row * H);
  uint4 v[VPL];
#pragma unroll
  for (int i = 0; i < VPL; ++i) v[i] = hr[i * 32 + lane];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const uint32_t u[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
    if (sizeof(T) == 2) {
      // squares rounded to bf16 two at a time (a bf16x2 multiply rounds the
      // exact product, as the fp32 multiply and round would), summed in
      // element order
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const __nv_bfloat162 e2 = *reinterpret_cast<const __nv_bfloat162*>(&u[q]);
        const __nv_bfloat162 sq = __hmul2(e2, e2);
        const uint32_t sw = *reinterpret_cast<const uint32_t*>(&sq);
        ss += bf16_bits_lo(sw);
        ss += bf16_bits_hi(sw);
      }
    } else {
#pragma unroll
      for (int j = 0; j < V; ++j) {
        const float e = __uint_as_float(u[j]);
        ss += e * e;
      }
    }
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
  const float mean = Elt<T>::round(ss / (float)H);
  const float r = Elt<T>::round(1.0f / sqrtf(Elt<T>::round(mean + eps)));
  const uint4* wr = reinterpret_cast<const uint4*>(w);
  uint4* xr = reinterpret_cast<uint4*>(x + row * H);
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const uint4 wv = wr[i * 32 + lane];
    const uint32_t wu[4] = {wv.x, wv.y, wv.z, wv.w};
    const uint32_t hu[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
    uint32_t o[4];
    if (sizeof(T) == 2) {
      // bf16(w * bf16(h * r)), two elements per bf16x2 multiply (r is a bf16
      // value, so every product is rounded once from its exact value)
      const __nv_bfloat162 r2 = __float2bfloat162_rn(r);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const __nv_bfloat162 hn = __hmul2(*reinterpret_cast<const __nv_bfloat162*>(&hu[q]), r2);
        const __nv_bfloat162 p = __hmul2(*reinterpret_cast<const __nv_bfloat162*>(&wu[q]), hn);
        o[q] = *reinterpret_cast<const uint32_t*>(&p);
      }
    } else {
#pragma unroll
      for (int q = 0; q < 4; ++q)
        o[q] = __float_as_uint(__uint_as_float(wu[q]) * (__uint_as_float(hu[q]) * r));
    }
    xr[i * 32 + lane] = make_uint4(o[0], o[1], o[2], o[3]);
  }
  tl_end(tl, kTlNorm + 1);
}

// any H (multiple of 16 bytes / elements): one warp per row, strided, two passes
template <typename T>
__global__ void __launch_bounds__(256) k_rmsnorm_any(int64_t n, int H, const T* __restrict__ h,
                                                     const T* __restrict__ w, float eps,
                                                     T* __restrict__ x, uint64_t* tl) {
  const int lane = lane_id();
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + warp_id();
  tl_begin(tl, kTlNorm);
  if (row >= n) return;
  const T* hr = h + row * H;
  float ss = 0.f;
  for (int c = lane; c < H; c += 32) {
    const float e = Elt<T>::to_f(hr[c]);
    ss += Elt<T>::round(e * e);
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
  const float mean = Elt<T>::round(ss / (float)H);
  const float r = Elt<T>::round(1.0f / sqrtf(Elt<T>::round(mean + eps)));
  for (int c = lane; c < H; c += 32)
    x[row * H + c] = Elt<T>::from_f(Elt<T>::to_f(w[c]) * Elt<T>::round(Elt<T>::to_f(hr[c]) * r));
  tl_end(tl, kTlNorm + 1);
}

}  // namespace

void launch_rmsnorm(int dtype, int64_t n, int hidden, const void* h, const void* w, float eps,
                    void* x, uint64_t* tl, cudaStream_t st) {
  if (n <= 0) return;
  const unsigned grid = (unsigned)((n + 7) / 8);
  if (dtype == kBF16) {
    auto hb = static_cast<const __nv_bfloat16*>(h);
    auto wb = static_cast<const __nv_bfloat16*>(w);
    auto xb = static_cast<__nv_bfloat16*>(x);
    if (hidden == 1024)
      k_rmsnorm<__nv_bfloat16, 4><<<grid, 256, 0, st>>>(n, hidden, hb, wb, eps, xb, tl);
    else if (hidden == 4096)
      k_rmsnorm<__nv_bfloat16, 16><<<grid, 256, 0, st>>>(n, hidden, hb, wb, eps, xb, tl);
    else
      k_rmsnorm_any<__nv_bfloat16><<<grid, 256, 0, st>>>(n, hidden, hb, wb, eps, xb, tl);
  } else {
    k_rmsnorm_any<float><<<grid, 256, 0, st>>>(n, hidden, static_cast<const float*>(h),
                                                static_cast<const float*>(w), eps,
                                                static_cast<float*>(x), tl);
  }
}

}  // namespace mep
