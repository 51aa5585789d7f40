// Shared pieces of the lm_head CE kernels and the forward statistics kernel.
//
// Forward (this file): persistent tcgen05 GEMM, logits tile = X[tok,:] . W[v,:]
// in TMEM, folded by the epilogue into online (max, sum-exp, entropy numerator,
// argmax, target logit) per token over a vocab slab. Replaces the reference's
// pass-1 cuBLAS GEMM + lm_head_piece_kernel MODE 0 (solution/ops.py:216-251,
// solution/kernels.py:480-516). The backward lives in lmce_bwd.cuh.
//
// CTA layout (192 threads, one CTA per SM), shared with the backward kernel:
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
constexpr int BN = 256;           // UMMA N (vocab or hidden columns)
constexpr int BK = 64;            // 64 x 16-bit = one 128-byte swizzle row
constexpr int UMMA_K = 16;        // K per tcgen05.mma of kind::f16
constexpr int NUM_THREADS = 192;  // 6 warps
constexpr int EPI_THREADS = 128;
constexpr int EPI_THREAD0 = 64;   // first epilogue thread (warp 2, lane 0)
constexpr uint32_t TMEM_COLS = 2 * BN;
constexpr float LOG2E = 1.4426950408889634f;
constexpr float LN2 = 0.6931471805599453f;
constexpr float NEG_BIG = -1.0e30f;  // finite "minus infinity" for running maxima

constexpr int MN_BOX_BYTES = 64 * BK * 2;     // one {64 MN, 64 K} TMA box of an MN-major operand

// Tile geometry. Single CTA: a 128 x 256 output tile, the CTA holds 128 A rows and
// 256 B rows per k-block of 64 (48 KB stages, 4 of them). Pair (cta_group::2): a 256 x 256
// output tile over two CTAs; each CTA holds 128 A rows and 128 B rows of K = 128 per stage
// (64 KB stages, 3 of them), each operand loaded as one {64, 128, 2} box of a 3-D view
// (256 contiguous bytes per row; see pair_operand_desc), and 128 accumulator lanes; the
// leader issues the UMMAs.
template <bool PAIR>
struct TileCfg {
  static constexpr int TILE_M = PAIR ? 2 * BM : BM;     // output rows per tile
  static constexpr int B_ROWS = PAIR ? BN / 2 : BN;     // B rows staged by one CTA
  static constexpr int KB = PAIR ? 2 * BK : BK;         // K per stage
  static constexpr int A_BYTES = BM * KB * 2;           // 16 KB (one CTA) or 32 KB (pair)
  static constexpr int B_BYTES = B_ROWS * KB * 2;       // 32 KB
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = PAIR ? 3 : 4;
  static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 /*align slack*/ + 1024 /*barriers, ring*/;
  static constexpr int CTAS = PAIR ? 2 : 1;
};

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

struct StatsParams {
  int M;                    // tokens
  int N;                    // vocab rows of this shard
  int K;                    // hidden
  int n_slabs;              // vocab slabs per token block
  const int64_t* labels;    // token labels (global vocab ids, -100 = ignore)
  int64_t label_off;        // first global vocab id of this shard
  Part* parts;              // out [M][n_slabs]
  int* err;                 // device error word
  unsigned long long timeout_ns;
};

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

// Named barrier over the 128 epilogue threads (warps 2..5); barrier 0 is __syncthreads.
__device__ __forceinline__ void epilogue_bar() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

// Named barrier ID among COUNT threads (the epilogue warps of a kernel, or a subset).
template <int ID, int COUNT>
__device__ __forceinline__ void named_bar() {
  asm volatile("bar.sync %0, %1;" ::"n"(ID), "n"(COUNT) : "memory");
}

// named_bar that also returns the AND of `pred` over its COUNT threads (one answer for all).
template <int ID, int COUNT>
__device__ __forceinline__ bool named_bar_all(bool pred) {
  uint32_t out;
  asm volatile(
      "{\n\t.reg .pred pi, po;\n\t"
      "setp.ne.u32 pi, %1, 0;\n\t"
      "bar.red.and.pred po, %2, %3, pi;\n\t"
      "selp.u32 %0, 1, 0, po;\n\t}"
      : "=r"(out)
      : "r"(static_cast<uint32_t>(pred)), "n"(ID), "n"(COUNT)
      : "memory");
  return out != 0;
}

// ------------------------------------------------------- operand staging ---

// TMA loads of one k-block of the A (BM rows) or B (BN rows) operand into a stage.
// K-major: one box {64 K, ROWS} at (k0, row0). MN-major: ROWS/64 boxes {64 MN, 64 K}
// at (row0 + 64 i, k0), placed MN_BOX_BYTES apart.
template <int ROWS>
__device__ __forceinline__ void load_operand(uint8_t* dst, const CUtensorMap* map, uint64_t* bar, bool mn_major,
                                             int row0, int k0) {
  if (!mn_major) {
    tma_load_2d(dst, map, bar, k0, row0);
  } else {
#pragma unroll
    for (int i = 0; i < ROWS / 64; ++i) tma_load_2d(dst + i * MN_BOX_BYTES, map, bar, row0 + 64 * i, k0);
  }
}

// MN-major operand through a 3-D tensor map (one TMA instruction for all ROWS / 64
// blocks; same shared-memory image as load_operand with mn_major = true).
template <int ROWS>
__device__ __forceinline__ void load_operand_mn3(uint8_t* dst, const CUtensorMap* map, uint64_t* bar, int row0,
                                                 int k0) {
  tma_load_3d(dst, map, bar, 0, k0, row0 / 64);
}

// Descriptor of UMMA k-step k (0..7, K = 16 each) of a 128-row operand staged by one
// {64, 128, 2} box: K = 128 per stage. K-major: two 16 KB blocks of 128 rows x 64 k (rows
// 128 bytes apart, SBO 1024 per 8 rows), k-step k in block k / 4 at 32 bytes per step.
// MN-major: two 64-element MN blocks 16 KB apart (LBO) of 128 k-rows of 128 bytes (SBO 1024
// per 8 k-rows), k-step k at 16 k-rows = 2048 bytes per step.
constexpr int BLOCK128_BYTES = BM * BK * 2;  // one 64-element block of a 128-row operand: 16 KB
__device__ __forceinline__ uint64_t pair_operand_desc(uint32_t base, bool mn_major, int k) {
  return mn_major ? smem_desc_sw128(base + k * (UMMA_K * 128), BLOCK128_BYTES, 1024)
                  : smem_desc_sw128(base + (k >> 2) * BLOCK128_BYTES + (k & 3) * (UMMA_K * 2), 16, 1024);
}

// Descriptor of UMMA k-step k (K = 16) inside a staged operand. K-major: rows of
// 128 bytes in 8-row swizzle atoms (SBO 1024), k advances 32 bytes within the row.
// MN-major: K rows of 128 bytes (8-row groups, SBO 1024), 64-wide MN blocks
// MN_BOX_BYTES apart (LBO), k advances 16 K rows = 2048 bytes.
__device__ __forceinline__ uint64_t operand_desc(uint32_t base, bool mn_major, int k) {
  return mn_major ? smem_desc_sw128(base + k * (UMMA_K * 128), MN_BOX_BYTES, 1024)
                  : smem_desc_sw128(base + k * (UMMA_K * 2), 16, 1024);
}

// ------------------------------------------------------- statistics kernel ---

// Work units: (token block, vocab slab), token-block-fastest, so the CTAs running
// at the same time read the same W tiles (shared through L2) and W streams from
// HBM about once. A slab is a run of consecutive 256-row vocab tiles whose
// statistics each epilogue thread carries in registers.
struct StatsSchedule {
  int num_m, num_n, n_slabs, total, num_kb;
  __device__ __forceinline__ void init(const StatsParams& p, int tile_m, int kb) {
    num_m = (p.M + tile_m - 1) / tile_m;
    num_n = (p.N + BN - 1) / BN;
    num_kb = (p.K + kb - 1) / kb;
    n_slabs = p.n_slabs;
    total = num_m * n_slabs;
  }
  __device__ __forceinline__ void unit(int u, int& m_blk, int& n_begin, int& n_end, int& slab) const {
    m_blk = u % num_m;
    slab = u / num_m;
    n_begin = static_cast<int>((static_cast<long long>(slab) * num_n) / n_slabs);
    n_end = static_cast<int>((static_cast<long long>(slab + 1) * num_n) / n_slabs);
  }
};

template <bool BF16, bool PAIR>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    lmce_stats_kernel(const __grid_constant__ CUtensorMap map_x, const __grid_constant__ CUtensorMap map_w,
                      const StatsParams p) {
  using C = TileCfg<PAIR>;
  constexpr int STAGES = C::STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + STAGES * C::STAGE_BYTES);
  uint64_t* empty_bar = full_bar + STAGES;
  uint64_t* tfull_bar = empty_bar + STAGES;
  uint64_t* tempty_bar = tfull_bar + 2;
  uint64_t* drain_bar = tempty_bar + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(drain_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = __shfl_sync(0xffffffffu, threadIdx.x / 32, 0);
  const int lane = threadIdx.x & 31;
  const uint32_t rank = PAIR ? cluster_rank() : 0u;          // 0 = leader (issues the UMMAs)
  const int unit0 = PAIR ? static_cast<int>(cluster_id_x()) : static_cast<int>(blockIdx.x);
  const int unit_step = PAIR ? static_cast<int>(cluster_count_x()) : static_cast<int>(gridDim.x);

  StatsSchedule sch;
  sch.init(p, C::TILE_M, C::KB);
  if (unit0 >= sch.total) return;  // uniform for the CTA (and for both CTAs of a pair)

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull_bar[b], 1);
      mbar_init(&tempty_bar[b], C::CTAS * EPI_THREADS);
    }
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&map_x);
    tma_prefetch_desc(&map_w);
  }
  if (warp == 1) {
    if constexpr (PAIR) {
      tmem_alloc_pair(tmem_holder, TMEM_COLS);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(tmem_holder, TMEM_COLS);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  __syncthreads();
  if constexpr (PAIR) cluster_sync();  // peer barriers initialised before any remote arrive / copy
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
      for (int u = unit0; ok && u < sch.total; u += unit_step) {
        int m_blk, n0, n1, slab;
        sch.unit(u, m_blk, n0, n1, slab);
        for (int n_blk = n0; ok && n_blk < n1; ++n_blk) {
          for (int kb = 0; kb < sch.num_kb; ++kb) {
            if (!mbar_wait(&empty_bar[stage], phase ^ 1u, abort_flag, tlimit)) {
              ok = false;
              break;
            }
            uint8_t* sa = smem + stage * C::STAGE_BYTES;
            uint8_t* sb = sa + C::A_BYTES;
            const int k0 = kb * C::KB;
            if constexpr (PAIR) {
              // both CTAs' copies count on the leader's full barrier; one {64, 128, 2} box per
              // operand: this CTA's 128 rows x two k-blocks
              if (rank == 0) mbar_arrive_expect_tx(&full_bar[stage], 2 * C::STAGE_BYTES);
              const uint32_t fb = mapa_shared(smem_u32(&full_bar[stage]), 0);
              tma_load_3d_pair(sa, &map_x, fb, 0, m_blk * C::TILE_M + BM * static_cast<int>(rank), 2 * kb);
              tma_load_3d_pair(sb, &map_w, fb, 0, n_blk * BN + C::B_ROWS * static_cast<int>(rank), 2 * kb);
            } else {
              mbar_arrive_expect_tx(&full_bar[stage], C::STAGE_BYTES);
              load_operand<BM>(sa, &map_x, &full_bar[stage], false, m_blk * BM, k0);
              load_operand<BN>(sb, &map_w, &full_bar[stage], false, n_blk * BN, k0);
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
        if (!PAIR || rank == 0) {
          // Drain: wait (bounded) for the copies counted on this CTA's barriers.
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
    }
  } else if (warp == 1) {
    // -------------------------------------------------------- UMMA issuer ---
    if (lane == 0 && rank == 0) {
      constexpr uint32_t idesc = make_idesc_f16(BF16, false, false, C::TILE_M, BN);
      const uint32_t peer_empty = PAIR ? mapa_shared(smem_u32(empty_bar), 1) : 0u;
      const uint32_t peer_tfull = PAIR ? mapa_shared(smem_u32(tfull_bar), 1) : 0u;
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int u = unit0; ok && u < sch.total; u += unit_step) {
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
            const uint32_t sa = smem_u32(smem + stage * C::STAGE_BYTES);
#pragma unroll
            for (int k = 0; k < C::KB / UMMA_K; ++k) {
              if constexpr (PAIR)
                umma_f16_ss_pair(d_tmem, pair_operand_desc(sa, false, k), pair_operand_desc(sa + C::A_BYTES, false, k),
                                 idesc, (kb | k) != 0 ? 1u : 0u);
              else
                umma_f16_ss(d_tmem, operand_desc(sa, false, k), operand_desc(sa + C::A_BYTES, false, k), idesc,
                            (kb | k) != 0 ? 1u : 0u);
            }
            if constexpr (PAIR) {
              umma_commit_pair(smem_u32(&empty_bar[stage]));
              umma_commit_pair(peer_empty + 8u * stage);
            } else {
              umma_commit(&empty_bar[stage]);
            }
            if (++stage == STAGES) {
              stage = 0;
              phase ^= 1u;
            }
          }
          if (!ok) break;
          if constexpr (PAIR) {
            umma_commit_pair(smem_u32(&tfull_bar[acc]));
            umma_commit_pair(peer_tfull + 8u * acc);
          } else {
            umma_commit(&tfull_bar[acc]);
          }
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
      if constexpr (PAIR)
        umma_commit_pair(smem_u32(drain_bar));
      else
        umma_commit(drain_bar);
      volatile int no_abort = 0;
      mbar_wait(drain_bar, 0, &no_abort, tlimit);
    }
  } else {
    // ---------------------------------------------------------- epilogue ---
    const int q = warp & 3;  // TMEM lane quadrant this warp may access
    const int r_in_tile = BM * static_cast<int>(rank) + q * 32 + lane;
    const uint32_t lane_base = static_cast<uint32_t>(q * 32) << 16;
    const uint32_t leader_tempty = PAIR ? mapa_shared(smem_u32(tempty_bar), 0) : 0u;
    int acc = 0;
    uint32_t acc_phase = 0;
    bool ok = true;

    for (int u = unit0; ok && u < sch.total; u += unit_step) {
      int m_blk, n0, n1, slab;
      sch.unit(u, m_blk, n0, n1, slab);
      const int row = m_blk * C::TILE_M + r_in_tile;

      float st_m = NEG_BIG, st_s = 0.f, st_w = 0.f, st_best = -INFINITY, st_zy = -INFINITY;
      int st_idx = 0x7fffffff;
      int lbl = -1;  // label local to the shard
      if (row < p.M) {
        const int64_t y = p.labels[row];
        const int64_t yl = y - p.label_off;
        lbl = (y != -100 && yl >= 0 && yl < p.N) ? static_cast<int>(yl) : -1;
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
          __syncwarp();
          tmem_ld_32x32b_x32(taddr + c * 32, raw);
          tmem_ld_wait(raw);
          const int col0 = n_blk * BN + c * 32;
          // Logits rounded to the input dtype, like the reference's fp16 GEMM output. All
          // statistics use the rounded values: for bf16 the rounding alone moves the entropy by
          // up to ~0.5%, so skipping it would leave the reference's definition.
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = round_to_input<BF16>(__uint_as_float(raw[j]));
          if (col0 + 32 > p.N) {
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (col0 + j >= p.N) v[j] = NEG_BIG;
          }
          float cmax = v[0];
#pragma unroll
          for (int j = 1; j < 32; ++j) cmax = fmaxf(cmax, v[j]);
          if (cmax > st_best) {  // strict: earlier columns keep ties
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
        }
        tc_fence_before();
        if constexpr (PAIR)
          mbar_arrive_cluster(leader_tempty + 8u * acc);
        else
          mbar_arrive(&tempty_bar[acc]);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }

      if (ok && row < p.M) {
        Part* dst = p.parts + static_cast<size_t>(row) * p.n_slabs + slab;
        float2* d2 = reinterpret_cast<float2*>(dst);
        d2[0] = make_float2(st_m, st_s);
        d2[1] = make_float2(st_w, st_best);
        d2[2] = make_float2(__int_as_float(st_idx), st_zy);
      }
    }
    if (!ok) {
      raise_error(p.err, ERR_TIMEOUT);
      *abort_flag = 1;
    }
  }

  tc_fence_before();
  __syncthreads();
  if constexpr (PAIR) cluster_sync();  // the leader's UMMAs into the peer's TMEM have drained
  tc_fence_after();
  if (warp == 1) {
    __syncwarp();
    if constexpr (PAIR)
      tmem_dealloc_pair(tmem_base, TMEM_COLS);
    else
      tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

}  // namespace lmce
