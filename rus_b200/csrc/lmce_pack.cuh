// Packing around the head, on the device (the label shift, keep mask and compaction
// before the head, solution/ops.py:1107-1127, and the scatter of its per-token outputs
// back to [B, S] after it, ops.py:1151-1164), in two launches each and with the kept
// count left on the device.
#pragma once

#include <cstdint>

namespace lmce {

constexpr int PACK_THREADS = 1024;

// Exclusive prefix sum of `c` over the block (PACK_THREADS threads); *total gets the sum.
__device__ __forceinline__ int block_exclusive_scan(int c, int* total) {
  __shared__ int s_warp[PACK_THREADS / 32];
  const int lane = threadIdx.x & 31, w = threadIdx.x / 32;
  int incl = c;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const int o = __shfl_up_sync(0xffffffffu, incl, off);
    if (lane >= off) incl += o;
  }
  if (lane == 31) s_warp[w] = incl;
  __syncthreads();
  if (w == 0) {
    int v = lane < PACK_THREADS / 32 ? s_warp[lane] : 0;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int o = __shfl_up_sync(0xffffffffu, v, off);
      if (lane >= off) v += o;
    }
    s_warp[lane] = v;  // inclusive warp totals
  }
  __syncthreads();
  const int excl = incl - c + (w > 0 ? s_warp[w - 1] : 0);
  *total = s_warp[PACK_THREADS / 32 - 1];
  __syncthreads();  // s_warp may be reused by the caller's next scan
  return excl;
}

// Shifted label of position t = b * S + s: labels[b, s + 1], -100 for the last position.
__device__ __forceinline__ int64_t shifted_label(const int64_t* labels, int64_t t, int64_t S) {
  return (t % S) < S - 1 ? labels[t + 1] : static_cast<int64_t>(-100);
}

// One block: keep = attended | shifted label != -100 (position 0 of every row when
// nothing is kept); kept positions compacted in order. Each thread owns a contiguous
// run of positions; row_lengths (zeroed by the caller) get one atomic add per run and row.
__global__ void __launch_bounds__(PACK_THREADS) pack_tokens_kernel(const int64_t* __restrict__ labels,
                                                                   const int64_t* __restrict__ mask, int64_t B,
                                                                   int64_t S, int64_t* __restrict__ shift_out,
                                                                   int64_t* __restrict__ idx_out,
                                                                   int* __restrict__ row_lengths, int* count) {
  const int64_t total = B * S;
  const int64_t per = (total + PACK_THREADS - 1) / PACK_THREADS;
  const int64_t t0 = threadIdx.x * per;
  const int64_t t1 = t0 + per < total ? t0 + per : total;
  int c = 0;
  // no mask: every position is attended (the reference's default, ops.py:1104-1105)
  for (int64_t t = t0; t < t1; ++t)
    c += ((mask == nullptr || mask[t] != 0) || shifted_label(labels, t, S) != -100) ? 1 : 0;
  int kept_total = 0;
  int pos = block_exclusive_scan(c, &kept_total);
  const bool none = kept_total == 0;  // the reference keeps position 0 of every row then
  int run_row = -1, run_n = 0;
  for (int64_t t = t0; t < t1; ++t) {
    const int64_t y = shifted_label(labels, t, S);
    const bool keep = none ? (t % S) == 0 : ((mask == nullptr || mask[t] != 0) || y != -100);
    if (!keep) continue;
    const int row = static_cast<int>(t / S);
    if (none) pos = row;  // one kept position per row, in row order
    shift_out[pos] = y;
    idx_out[pos] = t;
    ++pos;
    if (row != run_row) {
      if (run_n) atomicAdd(&row_lengths[run_row], run_n);
      run_row = row;
      run_n = 0;
    }
    ++run_n;
  }
  if (run_n) atomicAdd(&row_lengths[run_row], run_n);
  if (threadIdx.x == 0) *count = none ? static_cast<int>(B) : kept_total;
}

// packed[i] = hidden[idx[i]] for i < *count (rows of `vec` 16-byte units).
__global__ void pack_rows_kernel(const uint4* __restrict__ hidden, int vec, const int64_t* __restrict__ idx,
                                 const int* __restrict__ count, uint4* __restrict__ packed) {
  const long long total = static_cast<long long>(*count) * vec;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long r = i / vec;
    packed[i] = hidden[idx[r] * vec + (i - r * vec)];
  }
}

// One block: every position gets nll 0, argmax 0 and the mean entropy of the kept
// tokens (0 when there are none); the kept ones are overwritten by scatter_outputs_kernel.
__global__ void __launch_bounds__(PACK_THREADS) fill_outputs_kernel(const float* __restrict__ entropy,
                                                                    const int* __restrict__ count, int64_t total,
                                                                    float* __restrict__ full_nll,
                                                                    float* __restrict__ full_ent,
                                                                    int64_t* __restrict__ full_arg) {
  __shared__ float s_part[PACK_THREADS / 32];
  const int n = *count;
  float acc = 0.f;
  for (int i = threadIdx.x; i < n; i += PACK_THREADS) acc += entropy[i];
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
  if ((threadIdx.x & 31) == 0) s_part[threadIdx.x / 32] = acc;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = s_part[threadIdx.x];
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
    if (threadIdx.x == 0) s_part[0] = n > 0 ? v / static_cast<float>(n) : 0.f;
  }
  __syncthreads();
  const float mean = s_part[0];
  for (int64_t t = threadIdx.x; t < total; t += PACK_THREADS) {
    full_nll[t] = 0.f;
    full_ent[t] = mean;
    full_arg[t] = 0;
  }
}

__global__ void scatter_outputs_kernel(const float* __restrict__ nll, const float* __restrict__ entropy,
                                       const int64_t* __restrict__ argmax, const int64_t* __restrict__ idx,
                                       const int* __restrict__ count, float* __restrict__ full_nll,
                                       float* __restrict__ full_ent, int64_t* __restrict__ full_arg) {
  const int n = *count;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const int64_t t = idx[i];
    full_nll[t] = nll[i];
    full_ent[t] = entropy[i];
    full_arg[t] = argmax[i];
  }
}

}  // namespace lmce
