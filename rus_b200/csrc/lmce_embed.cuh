// Gradient of a tied input embedding added into the head's dW (the weight's two
// gradient contributions summed in one buffer, no second [V, H] tensor): for token
// positions i with id v in this shard, dW[v, :] += d_embed[i, :]. Positions are
// grouped by id with a counting sort (histogram, scan, scatter); each group is summed
// in fp64 together with the head's value and rounded once to the weight dtype. fp16
// values (11-bit significands, exponents within 2^-24 .. 2^15) add exactly in fp64 for
// up to 8192 positions per id, so the result does not depend on the order the scatter
// produced; bf16 sums are exact unless their magnitudes span more than 2^45.
#pragma once

#include <cstdint>

#include "lmce_engine.cuh"
#include "lmce_pack.cuh"

namespace lmce {

constexpr int EMB_COLS = 256;  // columns per warp task (8 per lane)

template <bool BF16>
__device__ __forceinline__ uint32_t pack2_from_double(double a, double b) {
  if constexpr (BF16) {
    const __nv_bfloat16 x = __double2bfloat16(a), y = __double2bfloat16(b);
    return static_cast<uint32_t>(__bfloat16_as_ushort(x)) | (static_cast<uint32_t>(__bfloat16_as_ushort(y)) << 16);
  } else {
    const __half x = __double2half(a), y = __double2half(b);
    return static_cast<uint32_t>(__half_as_ushort(x)) | (static_cast<uint32_t>(__half_as_ushort(y)) << 16);
  }
}

__global__ void emb_hist_kernel(const int64_t* __restrict__ ids, int64_t n, int64_t v_off, int v_local,
                                int* __restrict__ counts) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t v = ids[i] - v_off;
    if (v >= 0 && v < v_local) atomicAdd(&counts[v], 1);
  }
}

// One block: offsets[v] = sum of counts[0, v); cursor = offsets; the ids that occur,
// in order, in used[0, *n_used).
__global__ void __launch_bounds__(PACK_THREADS) emb_scan_kernel(const int* __restrict__ counts, int v_local,
                                                                int* __restrict__ offsets, int* __restrict__ cursor,
                                                                int* __restrict__ used, int* __restrict__ n_used) {
  const int per = (v_local + PACK_THREADS - 1) / PACK_THREADS;
  const int v0 = threadIdx.x * per;
  const int v1 = min(v0 + per, v_local);
  int c = 0, u = 0;
  for (int v = v0; v < v1; ++v) {
    c += counts[v];
    u += counts[v] > 0 ? 1 : 0;
  }
  int total = 0, total_used = 0;
  int pos = block_exclusive_scan(c, &total);
  int upos = block_exclusive_scan(u, &total_used);
  for (int v = v0; v < v1; ++v) {
    offsets[v] = pos;
    cursor[v] = pos;
    pos += counts[v];
    if (counts[v] > 0) used[upos++] = v;
  }
  if (threadIdx.x == 0) *n_used = total_used;
}

__global__ void emb_scatter_kernel(const int64_t* __restrict__ ids, int64_t n, int64_t v_off, int v_local,
                                   int* __restrict__ cursor, int* __restrict__ order) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t v = ids[i] - v_off;
    if (v >= 0 && v < v_local) order[atomicAdd(&cursor[v], 1)] = static_cast<int>(i);
  }
}

// One warp per (id that occurs, 256-column block): dW row block += fp64 sum of its
// positions' d_embed rows. The grid covers an upper bound of the ids that occur.
template <bool BF16>
__global__ void emb_accumulate_kernel(const uint4* __restrict__ d_embed, int h, const int* __restrict__ used,
                                      const int* __restrict__ n_used, const int* __restrict__ counts,
                                      const int* __restrict__ offsets, const int* __restrict__ order,
                                      uint4* __restrict__ d_weight) {
  const int nblk = (h + EMB_COLS - 1) / EMB_COLS;
  const long long task = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) / 32;
  const int lane = threadIdx.x & 31;
  if (task >= static_cast<long long>(*n_used) * nblk) return;
  const int v = used[task / nblk];
  const int cb = static_cast<int>(task % nblk);
  const int k = counts[v];
  const int col = cb * EMB_COLS + lane * 8;
  if (col >= h) return;
  const int vec = h / 8;  // 16-byte units per row
  double acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  const int o = offsets[v];
  for (int j = 0; j < k; ++j) {
    const uint4 u = d_embed[static_cast<long long>(order[o + j]) * vec + col / 8];
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      float a, b;
      if constexpr (BF16) {
        a = __uint_as_float(w[q] << 16);
        b = __uint_as_float(w[q] & 0xffff0000u);
      } else {
        const __half2 hv = *reinterpret_cast<const __half2*>(&w[q]);
        a = __low2float(hv);
        b = __high2float(hv);
      }
      acc[2 * q] += a;
      acc[2 * q + 1] += b;
    }
  }
  uint4* dst = d_weight + static_cast<long long>(v) * vec + col / 8;
  const uint4 cur = *dst;
  const uint32_t cw[4] = {cur.x, cur.y, cur.z, cur.w};
  uint32_t out[4];
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    float a, b;
    if constexpr (BF16) {
      a = __uint_as_float(cw[q] << 16);
      b = __uint_as_float(cw[q] & 0xffff0000u);
    } else {
      const __half2 hv = *reinterpret_cast<const __half2*>(&cw[q]);
      a = __low2float(hv);
      b = __high2float(hv);
    }
    // the head's value plus the embedding's sum, rounded once to the weight dtype
    out[q] = pack2_from_double<BF16>(acc[2 * q] + static_cast<double>(a), acc[2 * q + 1] + static_cast<double>(b));
  }
  *dst = make_uint4(out[0], out[1], out[2], out[3]);
}

// out[i] = weight[ids[i] - v_off] (zero rows for ids outside the shard); 16-byte units.
__global__ void emb_lookup_kernel(const uint4* __restrict__ weight, const int64_t* __restrict__ ids, int64_t n,
                                  int vec, int64_t v_off, int v_local, uint4* __restrict__ out) {
  const long long total = n * static_cast<long long>(vec);
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long r = i / vec;
    const int64_t v = ids[r] - v_off;
    out[i] = (v >= 0 && v < v_local) ? weight[v * vec + (i - r * vec)] : make_uint4(0u, 0u, 0u, 0u);
  }
}

}  // namespace lmce
