// Final RMSNorm fused with the packing gather in front of the head, and its backward fused
// with the scatter back to the unpacked rows (the reference normalises all rows with
// rms_norm_fwd before packing, solution/ops.py:824 with kernels.py:124-164, and
// backpropagates with rms_norm_bwd, ops.py:850 with kernels.py:167-190). One warp per row.
// Forward, per kept row: rstd = rsqrt(mean(h^2) + eps) in fp32; x = dtype(dtype(h * rstd) * w)
// (Qwen2RMSNorm's casting order). Backward: x_hat = h * rstd, wdy = w * dy,
// c = mean(x_hat * wdy), dh = (wdy - x_hat * c) * rstd.
#pragma once

#include <cstdint>

#include "lmce_engine.cuh"

namespace lmce {

template <bool BF16>
__device__ __forceinline__ void unpack8(const uint4& u, float* f) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    if constexpr (BF16) {
      f[2 * q] = __uint_as_float(w[q] << 16);
      f[2 * q + 1] = __uint_as_float(w[q] & 0xffff0000u);
    } else {
      const __half2 hv = *reinterpret_cast<const __half2*>(&w[q]);
      f[2 * q] = __low2float(hv);
      f[2 * q + 1] = __high2float(hv);
    }
  }
}

template <bool BF16>
__device__ __forceinline__ uint4 pack8(const float* f) {
  return make_uint4(pack2<BF16>(f[0], f[1]), pack2<BF16>(f[2], f[3]), pack2<BF16>(f[4], f[5]),
                    pack2<BF16>(f[6], f[7]));
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
  return v;
}

// x[i] = RMSNorm(h[idx[i]]) for i < n (idx NULL: row i), rstd[i] saved for the backward.
// `vec` 16-byte units (8 values) per row; a lane handles every 32nd unit.
template <bool BF16>
__global__ void rmsnorm_pack_kernel(const uint4* __restrict__ h, const uint4* __restrict__ w,
                                    const int64_t* __restrict__ idx, const int* __restrict__ count, int64_t n_max,
                                    int vec, float inv_cols, float eps, uint4* __restrict__ x,
                                    float* __restrict__ rstd_out) {
  const long long n = count ? *count : n_max;
  const int lane = threadIdx.x & 31;
  for (long long r = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) / 32; r < n;
       r += static_cast<long long>(gridDim.x) * blockDim.x / 32) {
    const uint4* src = h + (idx ? idx[r] : r) * vec;
    float ss = 0.f;
    for (int c = lane; c < vec; c += 32) {
      float f[8];
      unpack8<BF16>(src[c], f);
#pragma unroll
      for (int j = 0; j < 8; ++j) ss = fmaf(f[j], f[j], ss);
    }
    const float rstd = rsqrtf(warp_sum(ss) * inv_cols + eps);
    if (lane == 0) rstd_out[r] = rstd;
    uint4* dst = x + r * vec;
    for (int c = lane; c < vec; c += 32) {
      float f[8], g[8];
      unpack8<BF16>(src[c], f);
      unpack8<BF16>(w[c], g);
#pragma unroll
      for (int j = 0; j < 8; ++j) f[j] = round_to_input<BF16>(f[j] * rstd) * g[j];
      dst[c] = pack8<BF16>(f);
    }
  }
}

// dh[idx[i]] = RMSNorm backward of dy[i] for i < n (idx NULL: row i); rows of dh that are
// not kept stay as the caller left them (zeroed).
template <bool BF16>
__global__ void rmsnorm_backward_kernel(const uint4* __restrict__ dy, const uint4* __restrict__ h,
                                        const uint4* __restrict__ w, const float* __restrict__ rstd_in,
                                        const int64_t* __restrict__ idx, const int* __restrict__ count,
                                        int64_t n_max, int vec, float inv_cols, uint4* __restrict__ dh) {
  const long long n = count ? *count : n_max;
  const int lane = threadIdx.x & 31;
  for (long long r = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) / 32; r < n;
       r += static_cast<long long>(gridDim.x) * blockDim.x / 32) {
    const long long t = idx ? idx[r] : r;
    const uint4* hs = h + t * vec;
    const uint4* dys = dy + r * vec;
    const float rstd = rstd_in[r];
    float dot = 0.f;
    for (int c = lane; c < vec; c += 32) {
      float a[8], g[8], d[8];
      unpack8<BF16>(hs[c], a);
      unpack8<BF16>(w[c], g);
      unpack8<BF16>(dys[c], d);
#pragma unroll
      for (int j = 0; j < 8; ++j) dot = fmaf(a[j] * rstd, g[j] * d[j], dot);
    }
    const float cmean = warp_sum(dot) * inv_cols;
    uint4* out = dh + t * vec;
    for (int c = lane; c < vec; c += 32) {
      float a[8], g[8], d[8];
      unpack8<BF16>(hs[c], a);
      unpack8<BF16>(w[c], g);
      unpack8<BF16>(dys[c], d);
#pragma unroll
      for (int j = 0; j < 8; ++j) a[j] = (g[j] * d[j] - a[j] * rstd * cmean) * rstd;
      out[c] = pack8<BF16>(a);
    }
  }
}

}  // namespace lmce
