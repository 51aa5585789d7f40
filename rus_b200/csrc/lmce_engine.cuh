// Persistent tcgen05 GEMM engine with the four fused epilogues of the lm_head
// cross-entropy head.
//
//   STATS : logits tile = X[tok,:] . W[v,:]  ->  online (max, sum-exp, entropy
//           numerator, argmax, target logit) per token over a vocab slab.
//           Replaces the reference's pass-1 cuBLAS GEMM + lm_head_piece_kernel
//           MODE 0 (solution/ops.py:216-251, solution/kernels.py:480-516).
//   GRAD  : recomputed logits tile -> G = (softmax - onehot) * 2^15 in the input
//           dtype, written to a vocab-chunk workspace. Replaces the pass-2 GEMM +
//           lm_head_piece_kernel MODE 1 (ops.py:287-319, kernels.py:517-531).
//   DX    : dX_tok += G_chunk . W_chunk (fp32 accumulation across chunks, final
//           chunk scales by dnll / 2^15 and scatters rows to the token order).
//           Replaces ops.py:320 `d_h_prescaled.addmm_` and the rescale at 337-338.
//   DW    : dW_chunk = G_chunk^T . X_tok (absent in the reference, which returns
//           None for the weight at ops.py:339).
//
// CTA layout (192 threads, one CTA per SM):
//   warp 0      TMA producer (lane 0 issues), smem ring of STAGES stages
//   warp 1      TMEM allocator + UMMA issuer (lane 0 issues, commits)
//   warps 2..5  epilogue; warp w reads TMEM lanes 32*(w%4) .. +31, one token /
//               output row per thread
// Accumulators: two TMEM buffers of BN fp32 columns (128 lanes), so the epilogue
// of tile i overlaps the UMMAs of tile i+1.
#pragma once

#include "lmce_ptx.cuh"

namespace lmce {

constexpr int BM = 128;           // UMMA M (token rows or vocab rows)
constexpr int BK = 64;            // 64 x 16-bit = one 128-byte swizzle row
constexpr int UMMA_K = 16;        // K per tcgen05.mma of kind::f16
constexpr int NUM_THREADS = 192;  // 6 warps
constexpr int EPI_THREADS = 128;
constexpr float LOG2E = 1.4426950408889634f;
constexpr float LN2 = 0.6931471805599453f;
constexpr float NEG_BIG = -1.0e30f;  // finite "minus infinity" for running maxima

enum Kind : int { KIND_STATS = 0, KIND_GRAD = 1, KIND_DX = 2, KIND_DW = 3 };

enum : int {
  ERR_OK = 0,
  ERR_TIMEOUT = 4,
  ERR_LABEL = 5,
};

// One per-token partial of the online softmax statistics (24 bytes).
//   m    running max of the (dtype-rounded) logits
//   s    sum_v 2^((z_v - m) * log2 e)
//   w    sum_v 2^((z_v - m) * log2 e) * (z_v - m)      (entropy numerator, shifted)
//   best max logit seen, idx its lowest global vocab index
//   zy   target logit, -inf when the target is outside this partial's range
struct Part {
  float m, s, w, best;
  int idx;
  float zy;
};

struct EngineParams {
  int M;                    // rows of D (upper bound when count_dev drives M)
  int N;                    // columns of D
  int K;                    // contraction length (upper bound when count_dev drives K)
  const int* count_dev;     // GRAD/DX: device row count; DW: device K; else nullptr
  int b_off;                // GRAD: W row offset (chunk start); DX: W k offset (chunk start); DW: dW row offset
  int n_slabs;              // STATS: vocab slabs per row block
  int v_limit;              // STATS: V_local; GRAD/DW: valid vocab columns/rows of this chunk
  const int64_t* labels;    // STATS: token labels (global vocab ids, -100 = ignore)
  int64_t label_off;        // STATS: first global vocab id of this shard
  Part* parts;              // STATS: out [M][n_slabs]
  const int* lbl_lab;       // GRAD: per compact row, label local to the shard (-1: none)
  const float* lse_lab;     // GRAD: per compact row lse
  void* out;                // GRAD: G [.][ldo]; DX: final dX rows (dtype); DW: dW (dtype)
  float* out_f32;           // DX: final dX rows in fp32 (vocab-sharded runs)
  float* acc_f32;           // DX: running accumulator [rows][N] (compact order)
  const int* row_idx;       // DX: compact row -> token row
  int ldo;                  // leading dimension (elements) of out / out_f32 / acc_f32
  int first, last;          // DX: first / last vocab chunk
  const float* grad_loss;   // DX/DW: upstream gradient of the loss (device scalar, nullable)
  const float* denom;       // DX/DW: loss denominator (device scalar)
  float gscale;             // GRAD prescale, un-done in DX/DW
  int* err;                 // device error word
  unsigned long long timeout_ns;
};

template <int BN>
struct Shape {
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
};

template <int BN, int STAGES>
constexpr int engine_smem_bytes() {
  return STAGES * Shape<BN>::STAGE_BYTES + 1024 /*align slack*/ + 512 /*barriers*/;
}

// ------------------------------------------------------------- conversion ---

template <bool BF16>
__device__ __forceinline__ float round_to_input(float x) {
  if constexpr (BF16) {
    return __bfloat162float(__float2bfloat16_rn(x));
  } else {
    return __half2float(__float2half_rn(x));
  }
}

template <bool BF16>
__device__ __forceinline__ uint32_t pack2(float a, float b) {
  if constexpr (BF16) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  } else {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
}

// Store 32 consecutive floats as 32 dtype elements (4 x 16-byte stores).
template <bool BF16>
__device__ __forceinline__ void store32_dtype(void* dst, const float* v) {
  uint4* d = reinterpret_cast<uint4*>(dst);
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    uint4 u;
    u.x = pack2<BF16>(v[8 * q + 0], v[8 * q + 1]);
    u.y = pack2<BF16>(v[8 * q + 2], v[8 * q + 3]);
    u.z = pack2<BF16>(v[8 * q + 4], v[8 * q + 5]);
    u.w = pack2<BF16>(v[8 * q + 6], v[8 * q + 7]);
    d[q] = u;
  }
}

__device__ __forceinline__ void raise_error(int* err, int code) {
  if (err) atomicCAS(err, 0, code);
}

// ---------------------------------------------------------------- schedule ---

// Work decomposition shared by the three roles (each role walks it identically).
// STATS: unit = (row block, vocab slab), a run of consecutive vocab tiles whose
//        statistics are folded in registers; units are ordered row-block-fastest
//        so the CTAs running at the same time share W tiles through L2.
// Other kinds: unit = one output tile, ordered row-block-fastest.
template <int KIND, int BN>
struct Schedule {
  int num_m, num_n, n_slabs, total, num_kb;

  __device__ __forceinline__ void init(const EngineParams& p) {
    int rows = p.M;
    int kext = p.K;
    if (p.count_dev != nullptr) {
      const int c = *p.count_dev;
      if constexpr (KIND == KIND_DW) {
        kext = c;
      } else {
        rows = c;
      }
    }
    num_m = (rows + BM - 1) / BM;
    num_n = (p.N + BN - 1) / BN;
    num_kb = (kext + BK - 1) / BK;
    if constexpr (KIND == KIND_STATS) {
      n_slabs = p.n_slabs;
      total = num_m * n_slabs;
    } else {
      n_slabs = 1;
      total = num_m * num_n;
    }
  }

  __device__ __forceinline__ void unit(int u, int& m_blk, int& n_begin, int& n_end, int& slab) const {
    m_blk = u % num_m;
    if constexpr (KIND == KIND_STATS) {
      slab = u / num_m;
      n_begin = static_cast<int>((static_cast<long long>(slab) * num_n) / n_slabs);
      n_end = static_cast<int>((static_cast<long long>(slab + 1) * num_n) / n_slabs);
    } else {
      slab = 0;
      n_begin = u / num_m;
      n_end = n_begin + 1;
    }
  }
};

// ------------------------------------------------------------------ kernel ---

template <int KIND, int BN, bool A_MN, bool B_MN, bool BF16, int STAGES>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    lmce_gemm_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                     const EngineParams p) {
  static_assert(BN % 64 == 0 && BN <= 256, "BN must be a multiple of 64, at most 256");
  using S = Shape<BN>;
  constexpr uint32_t TMEM_COLS = 2 * BN;
  static_assert(TMEM_COLS == 128 || TMEM_COLS == 256 || TMEM_COLS == 512, "TMEM allocation must be a power of 2");

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + STAGES * S::STAGE_BYTES);
  uint64_t* empty_bar = full_bar + STAGES;
  uint64_t* tfull_bar = empty_bar + STAGES;
  uint64_t* tempty_bar = tfull_bar + 2;
  uint64_t* drain_bar = tempty_bar + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(drain_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = __shfl_sync(0xffffffffu, threadIdx.x / 32, 0);
  const int lane = threadIdx.x & 31;

  Schedule<KIND, BN> sch;
  sch.init(p);
  if (static_cast<int>(blockIdx.x) >= sch.total) return;  // uniform for the whole CTA

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull_bar[b], 1);
      mbar_init(&tempty_bar[b], EPI_THREADS);
    }
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&map_a);
    tma_prefetch_desc(&map_b);
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  const uint64_t tlimit = p.timeout_ns;

  if (warp == 0) {
    // ------------------------------------------------------ TMA producer ---
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int issued = 0;
      bool ok = true;
      for (int u = blockIdx.x; ok && u < sch.total; u += gridDim.x) {
        int m_blk, n0, n1, slab;
        sch.unit(u, m_blk, n0, n1, slab);
        for (int n_blk = n0; ok && n_blk < n1; ++n_blk) {
          for (int kb = 0; kb < sch.num_kb; ++kb) {
            if (!mbar_wait(&empty_bar[stage], phase ^ 1u, abort_flag, tlimit)) {
              ok = false;
              break;
            }
            uint8_t* sa = smem + stage * S::STAGE_BYTES;
            uint8_t* sb = sa + S::A_BYTES;
            mbar_arrive_expect_tx(&full_bar[stage], S::STAGE_BYTES);
            const int k0 = kb * BK;
            // A operand
            if constexpr (!A_MN) {
              tma_load_2d(sa, &map_a, &full_bar[stage], k0, m_blk * BM);
            } else {
#pragma unroll
              for (int i = 0; i < BM / 64; ++i)
                tma_load_2d(sa + i * (64 * BK * 2), &map_a, &full_bar[stage], m_blk * BM + 64 * i, k0);
            }
            // B operand
            if constexpr (!B_MN) {
              const int row0 = (KIND == KIND_GRAD ? p.b_off : 0) + n_blk * BN;
              tma_load_2d(sb, &map_b, &full_bar[stage], k0, row0);
            } else {
              const int kk = (KIND == KIND_DX ? p.b_off : 0) + k0;
#pragma unroll
              for (int i = 0; i < BN / 64; ++i)
                tma_load_2d(sb + i * (64 * BK * 2), &map_b, &full_bar[stage], n_blk * BN + 64 * i, kk);
            }
            ++issued;
            if (++stage == STAGES) {
              stage = 0;
              phase ^= 1u;
            }
          }
        }
      }
      if (!ok) {
        raise_error(p.err, ERR_TIMEOUT);
        *abort_flag = 1;
        // Drain: wait (bounded) for the copies this thread issued into each stage.
        const int outstanding = issued < STAGES ? issued : STAGES;
        for (int i = 1; i <= outstanding; ++i) {
          int s = stage - i;
          uint32_t ph = phase;
          if (s < 0) {
            s += STAGES;
            ph ^= 1u;
          }
          volatile int no_abort = 0;
          mbar_wait(&full_bar[s], ph, &no_abort, tlimit);
        }
      }
    }
  } else if (warp == 1) {
    // -------------------------------------------------------- UMMA issuer ---
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc_f16(BF16, A_MN, B_MN, BM, BN);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int u = blockIdx.x; ok && u < sch.total; u += gridDim.x) {
        int m_blk, n0, n1, slab;
        sch.unit(u, m_blk, n0, n1, slab);
        for (int n_blk = n0; ok && n_blk < n1; ++n_blk) {
          if (!mbar_wait(&tempty_bar[acc], acc_phase ^ 1u, abort_flag, tlimit)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
          for (int kb = 0; kb < sch.num_kb; ++kb) {
            if (!mbar_wait(&full_bar[stage], phase, abort_flag, tlimit)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t sa = smem_u32(smem + stage * S::STAGE_BYTES);
            const uint32_t sb = sa + S::A_BYTES;
#pragma unroll
            for (int k = 0; k < BK / UMMA_K; ++k) {
              uint64_t da, db;
              if constexpr (!A_MN) {
                da = smem_desc_sw128(sa + k * (UMMA_K * 2), 16, 1024);
              } else {
                da = smem_desc_sw128(sa + k * (UMMA_K * 128), 64 * BK * 2, 1024);
              }
              if constexpr (!B_MN) {
                db = smem_desc_sw128(sb + k * (UMMA_K * 2), 16, 1024);
              } else {
                db = smem_desc_sw128(sb + k * (UMMA_K * 128), 64 * BK * 2, 1024);
              }
              umma_f16_ss(d_tmem, da, db, idesc, (kb | k) != 0 ? 1u : 0u);
            }
            umma_commit(&empty_bar[stage]);
            if (++stage == STAGES) {
              stage = 0;
              phase ^= 1u;
            }
          }
          if (!ok) break;
          umma_commit(&tfull_bar[acc]);  // also fires when num_kb == 0 (no MMA issued)
          if (++acc == 2) {
            acc = 0;
            acc_phase ^= 1u;
          }
        }
      }
      if (!ok) {
        raise_error(p.err, ERR_TIMEOUT);
        *abort_flag = 1;
      }
      // Make sure every UMMA this thread issued has retired before TMEM is freed.
      umma_commit(drain_bar);
      volatile int no_abort = 0;
      mbar_wait(drain_bar, 0, &no_abort, tlimit);
    }
  } else {
    // ---------------------------------------------------------- epilogue ---
    const int q = warp & 3;  // TMEM lane quadrant this warp may access
    const int r_in_tile = q * 32 + lane;
    const uint32_t lane_base = static_cast<uint32_t>(q * 32) << 16;
    int acc = 0;
    uint32_t acc_phase = 0;
    bool ok = true;

    float dscale = 1.0f;
    if constexpr (KIND == KIND_DX || KIND == KIND_DW) {
      const float gl = p.grad_loss ? *p.grad_loss : 1.0f;
      dscale = gl / (*p.denom) / p.gscale;
    }
    const bool have_acc = sch.num_kb > 0;
    int rows_valid = p.M;
    if constexpr (KIND == KIND_GRAD || KIND == KIND_DX) {
      if (p.count_dev) rows_valid = *p.count_dev;
    }

    for (int u = blockIdx.x; ok && u < sch.total; u += gridDim.x) {
      int m_blk, n0, n1, slab;
      sch.unit(u, m_blk, n0, n1, slab);
      const int row = m_blk * BM + r_in_tile;

      // per-row state
      float st_m = NEG_BIG, st_s = 0.f, st_w = 0.f, st_best = -INFINITY, st_zy = -INFINITY;
      int st_idx = 0x7fffffff;
      int lbl = -1;       // STATS: label local to the shard; GRAD: label local to the chunk
      float lseL = 0.f;   // GRAD: lse * log2(e)
      if constexpr (KIND == KIND_STATS) {
        if (row < p.M) {
          const int64_t y = p.labels[row];
          const int64_t yl = y - p.label_off;
          lbl = (y != -100 && yl >= 0 && yl < p.v_limit) ? static_cast<int>(yl) : -1;
        }
      }
      if constexpr (KIND == KIND_GRAD) {
        if (row < rows_valid) {
          const int y = p.lbl_lab[row];
          lbl = y >= 0 ? y - p.b_off : -1;
          lseL = p.lse_lab[row] * LOG2E;
        }
      }

      for (int n_blk = n0; n_blk < n1; ++n_blk) {
        if (!mbar_wait(&tfull_bar[acc], acc_phase, abort_flag, tlimit)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t taddr = tmem_base + lane_base + static_cast<uint32_t>(acc * BN);

#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
          uint32_t raw[32];
          float v[32];
          tmem_ld_32x32b_x32(taddr + c * 32, raw);
          tmem_ld_wait(raw);
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = have_acc ? __uint_as_float(raw[j]) : 0.0f;
          const int col0 = n_blk * BN + c * 32;

          if constexpr (KIND == KIND_STATS) {
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = round_to_input<BF16>(v[j]);
            if (col0 + 32 > p.v_limit) {
#pragma unroll
              for (int j = 0; j < 32; ++j)
                if (col0 + j >= p.v_limit) v[j] = NEG_BIG;
            }
            float cmax = v[0];
#pragma unroll
            for (int j = 1; j < 32; ++j) cmax = fmaxf(cmax, v[j]);
            if (cmax > st_best) {
              int bj = 31;
#pragma unroll
              for (int j = 31; j >= 0; --j)
                if (v[j] == cmax) bj = j;
              st_best = cmax;
              st_idx = static_cast<int>(p.label_off) + col0 + bj;
            }
            if (cmax > st_m) {
              const float d = st_m - cmax;
              const float a = ex2_approx(d * LOG2E);
              st_w = a * fmaf(d, st_s, st_w);
              st_s = a * st_s;
              st_m = cmax;
            }
            const float mL = st_m * LOG2E;
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              const float e = ex2_approx(fmaf(v[j], LOG2E, -mL));
              st_s += e;
              st_w = fmaf(e, v[j] - st_m, st_w);
            }
            const unsigned rel = static_cast<unsigned>(lbl - col0);
            if (lbl >= 0 && rel < 32u) {
#pragma unroll
              for (int j = 0; j < 32; ++j)
                if (static_cast<unsigned>(j) == rel) st_zy = v[j];
            }
          } else if constexpr (KIND == KIND_GRAD) {
            float g[32];
            const bool row_ok = row < rows_valid;
            const unsigned rel = static_cast<unsigned>(lbl - col0);
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              const float z = round_to_input<BF16>(v[j]);
              float pr = ex2_approx(fmaf(z, LOG2E, -lseL));
              if (static_cast<unsigned>(j) == rel) pr -= 1.0f;
              g[j] = (row_ok && col0 + j < p.v_limit) ? pr * p.gscale : 0.0f;
            }
            if (row < p.M) {
              char* dst = reinterpret_cast<char*>(p.out) +
                          (static_cast<size_t>(row) * p.ldo + col0) * 2;
              store32_dtype<BF16>(dst, g);
            }
          } else if constexpr (KIND == KIND_DX) {
            if (row < rows_valid && col0 < p.N) {
              float o[32];
#pragma unroll
              for (int j = 0; j < 32; ++j) o[j] = v[j] * dscale;
              float* accp = p.acc_f32 + static_cast<size_t>(row) * p.ldo + col0;
              if (!p.first) {
#pragma unroll
                for (int j = 0; j < 32; j += 4) {
                  const float4 a4 = *reinterpret_cast<const float4*>(accp + j);
                  o[j] += a4.x;
                  o[j + 1] += a4.y;
                  o[j + 2] += a4.z;
                  o[j + 3] += a4.w;
                }
              }
              if (!p.last) {
#pragma unroll
                for (int j = 0; j < 32; j += 4)
                  *reinterpret_cast<float4*>(accp + j) = make_float4(o[j], o[j + 1], o[j + 2], o[j + 3]);
              } else {
                const size_t trow = static_cast<size_t>(p.row_idx[row]);
                if (p.out_f32 != nullptr) {
                  float* dst = p.out_f32 + trow * p.ldo + col0;
#pragma unroll
                  for (int j = 0; j < 32; j += 4)
                    *reinterpret_cast<float4*>(dst + j) = make_float4(o[j], o[j + 1], o[j + 2], o[j + 3]);
                }
                if (p.out != nullptr) {
                  char* dst = reinterpret_cast<char*>(p.out) + (trow * p.ldo + col0) * 2;
                  store32_dtype<BF16>(dst, o);
                }
              }
            }
          } else {  // KIND_DW
            if (row < p.v_limit && col0 < p.N) {
              float o[32];
#pragma unroll
              for (int j = 0; j < 32; ++j) o[j] = v[j] * dscale;
              char* dst = reinterpret_cast<char*>(p.out) +
                          ((static_cast<size_t>(p.b_off) + row) * p.ldo + col0) * 2;
              store32_dtype<BF16>(dst, o);
            }
          }
        }
        tc_fence_before();
        mbar_arrive(&tempty_bar[acc]);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }

      if constexpr (KIND == KIND_STATS) {
        if (ok && row < p.M) {
          Part* dst = p.parts + static_cast<size_t>(row) * p.n_slabs + slab;
          float2* d2 = reinterpret_cast<float2*>(dst);
          d2[0] = make_float2(st_m, st_s);
          d2[1] = make_float2(st_w, st_best);
          d2[2] = make_float2(__int_as_float(st_idx), st_zy);
        }
      }
    }
    if (!ok) {
      raise_error(p.err, ERR_TIMEOUT);
      *abort_flag = 1;
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, TMEM_COLS);
}

}  // namespace lmce
