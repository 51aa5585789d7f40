// Persistent backward of the lm_head CE head on CTA pairs (tcgen05 cta_group::2).
//
// Same work as lmce_bwd_kernel (recomputed logits -> G, dX and dW GEMMs), laid out
// so that the two CTAs of a cluster share every tile: the MMA is 256 x N, each CTA
// stages its 128 rows of A and N/2 rows of B (32 KB a k-block instead of 48 KB for a
// 128 x 256 tile on one SM), five stages deep. The token rows are the N dimension of
// the tiles that contract over them (a K-major B operand, any multiple of 16, used in
// steps of 64), so they are padded to 64, not to the M tile.
//   GT(c)   vocab block jv (M, 256) x row block i (N <= 256) of G^T = W_c . X_lab^T,
//           K = H: the epilogue forms G = (softmax - onehot) * 2^15 in the input dtype
//           and writes it, transposed through shared memory, to G buffer c % NUM_GBUF
//           as [row][vocab] (replaces the reference's pass-2 GEMM + lm_head_piece_kernel
//           MODE 1, solution/ops.py:287-319, solution/kernels.py:517-531)
//   DXT(c)  hidden block p (M) x row block i (N) of dX^T += W_c^T . G_c^T, K = chunk
//           width; fp32 accumulation in a [H][rows] buffer in chunk order; the last chunk
//           scales by grad_loss / denom / 2^15, transposes through shared memory and
//           scatters rows to token order (replaces ops.py:320 and 337-338)
//   DW(c)   vocab block jv (M) x hidden block p (N = 256) of dW = G_c^T . X_lab, K =
//           labelled tokens (new: the reference returns None for the weight, ops.py:339)
// The tile list, its order, the dependency counters and the fused cross-GPU exchange
// follow lmce_bwd_kernel; every count covers both CTAs of a pair (each CTA publishes
// its half). The pair leader (cluster rank 0) claims tickets, checks dependencies and
// hands each tile to both CTAs' schedule rings (the peer's through distributed shared
// memory); only the leader issues UMMAs. Every wait is bounded.
#pragma once

#include "lmce_bwd.cuh"

namespace lmce {

constexpr int P_STAGES = 5;
constexpr int P_THREADS = 320;  // warp 0 producer, warp 1 UMMA, warps 2-9 epilogue (two per TMEM lane quadrant)
constexpr int P_EPI = 256;
constexpr int P_A_BYTES = BM * BK * 2;                     // 128 rows x 64 k: 16 KB
constexpr int P_B_BYTES = BM * BK * 2;                     // up to 128 rows (N / 2) x 64 k: 16 KB
constexpr int P_STAGE_BYTES = P_A_BYTES + P_B_BYTES;       // 32 KB
constexpr int P_RB = 256;                                  // token rows per row block
constexpr int P_XPOSE_PITCH = 33 * 4;                      // fp32 32 x 32 transpose, conflict-free
constexpr int P_XPOSE_BYTES = 8 * 32 * P_XPOSE_PITCH;      // per-warp slices of the eight epilogue warps
constexpr int P_ROWDATA_BYTES = P_RB * 8;                  // per-tile lse * log2(e) and chunk-local label of 256 rows
// stages, 1 KB of barriers and ring, the staging slices, the row data, and 1 KB of slack
// for the 1024-byte alignment of the dynamic shared memory base
constexpr int PBWD_SMEM_BYTES = P_STAGES * P_STAGE_BYTES + 2048 + P_XPOSE_BYTES + P_ROWDATA_BYTES;
static_assert((2 * P_STAGES + 5 + 2 * SCHED_DEPTH) * 8 <= 256, "pair barriers end below the ring");
static_assert(32 * ROW_STAGE_PITCH <= 32 * P_XPOSE_PITCH, "16-bit staging fits a warp's slice");
static_assert(PBWD_SMEM_BYTES <= 227 * 1024, "dynamic shared memory of one CTA");

struct PairGeom {
  int n_lab, nrb, nh, C, vc, V, nX;
  bool dx, dw, xch;
  __device__ __forceinline__ int width(int c) const { return min(vc, V - c * vc); }
  __device__ __forceinline__ int nvb(int c) const { return (width(c) + 255) / 256; }
  __device__ __forceinline__ int nG(int c) const { return nvb(c) * nrb; }
  __device__ __forceinline__ int nDX() const { return dx ? nh * nrb : 0; }
  __device__ __forceinline__ int nDW(int c) const { return dw ? nvb(c) * nh : 0; }
  // N of a row-block tile: the block's rows rounded up to 64
  __device__ __forceinline__ int rows_n(int i) const {
    const int r = n_lab - i * P_RB;
    return r >= P_RB ? P_RB : ((r + 63) / 64) * 64;
  }
  __device__ __forceinline__ int num_kb(const BwdTile& t, int H) const {
    if (t.kind == BK_XCH) return 0;
    if (t.kind == BK_G) return (H + BK - 1) / BK;
    if (t.kind == BK_DX) return (width(t.chunk) + BK - 1) / BK;
    return (n_lab + BK - 1) / BK;
  }
};

__device__ __forceinline__ PairGeom make_pair_geom(const BwdParams& p) {
  PairGeom g;
  g.n_lab = *p.count;
  g.nrb = (g.n_lab + P_RB - 1) / P_RB;
  g.nh = (p.H + BN - 1) / BN;
  g.C = p.n_chunks;
  g.vc = p.v_chunk;
  g.V = p.V;
  g.dx = p.want_dx != 0;
  g.dw = p.want_dw != 0;
  g.xch = p.x_flags_mc != nullptr && g.dx;
  g.nX = g.xch ? g.nrb * ((p.x_hi - p.x_lo + XCH_COLS - 1) / XCH_COLS) : 0;
  return g;
}

// Decoder of the pair tile list (same segment order as TileCursor).
//   GT: m = row block (fastest: consecutive tiles share the W block), n = vocab block
//   DXT: m = row block (fastest: consecutive tiles share the W^T block), n = hidden block
//   DW: n = hidden block (fastest: consecutive tiles share the G columns), m = vocab block
//   XCH: m = row block, n = column piece
struct PairCursor {
  int seg;
  long long seg_start;

  __device__ __forceinline__ void init() {
    seg = 0;
    seg_start = 0;
  }

  __device__ __forceinline__ static bool segment(const PairGeom& g, int s, int& kind, int& chunk, int& count) {
    if (g.xch) {
      const int head = g.C >= 2 ? 3 * g.C - 3 : 1;
      if (s >= head) {
        const int u = s - head;
        chunk = g.C - 1;
        if (u == 0) {
          kind = BK_DX;
          count = g.nDX();
        } else if (u == 1) {
          kind = BK_XCH;
          count = g.nX;
        } else if (u <= 3) {
          kind = BK_DW;
          chunk = g.C - 4 + u;
          count = chunk >= 0 ? g.nDW(chunk) : 0;
        } else {
          return false;
        }
        return true;
      }
    }
    if (s == 0) {
      kind = BK_G;
      chunk = 0;
      count = g.nG(0);
      return true;
    }
    const int c = (s - 1) / 3, r = (s - 1) % 3;
    if (c >= g.C) return false;
    if (r == 0) {
      kind = BK_G;
      chunk = c + 1;
      count = c + 1 < g.C ? g.nG(c + 1) : 0;
    } else if (r == 1) {
      kind = BK_DX;
      chunk = c;
      count = g.nDX();
    } else {
      kind = BK_DW;
      chunk = c;
      count = g.nDW(c);
    }
    return true;
  }

  __device__ __forceinline__ bool decode(const PairGeom& g, long long t, BwdTile& out) {
    for (;;) {
      int kind, chunk, count;
      if (!segment(g, seg, kind, chunk, count)) return false;
      if (t < seg_start + count) {
        const int i = static_cast<int>(t - seg_start);
        out.kind = kind;
        out.chunk = chunk;
        if (kind == BK_DW) {
          out.n = i % g.nh;
          out.m = i / g.nh;
        } else {
          out.m = i % g.nrb;
          out.n = i / g.nrb;
        }
        return true;
      }
      seg_start += count;
      ++seg;
    }
  }
};

// Pair UMMA k-loop of one tile (leader only); the instruction descriptor is a template
// constant (see mma_tile). Both CTAs' empty barriers are signalled per stage.
template <bool BF16, bool A_MN, bool B_MN, int NCOLS>
__device__ __forceinline__ bool mma_tile_pair(uint8_t* smem, uint64_t* full_bar, uint64_t* empty_bar,
                                              uint32_t peer_empty, int nkb, uint32_t d_tmem, int& stage,
                                              uint32_t& phase, volatile int* abort_flag, uint64_t tlimit) {
  constexpr uint32_t idesc = make_idesc_f16(BF16, A_MN, B_MN, 2 * BM, NCOLS);
  for (int kb = 0; kb < nkb; ++kb) {
    if (!mbar_wait(&full_bar[stage], phase, abort_flag, tlimit)) return false;
    tc_fence_after();
    const uint32_t sa = smem_u32(smem + stage * P_STAGE_BYTES);
#pragma unroll
    for (int k = 0; k < BK / UMMA_K; ++k)
      umma_f16_ss_pair(d_tmem, operand_desc(sa, A_MN, k), operand_desc(sa + P_A_BYTES, B_MN, k), idesc,
                       (kb | k) != 0 ? 1u : 0u);
    umma_commit_pair(smem_u32(&empty_bar[stage]));
    umma_commit_pair(peer_empty + 8u * stage);
    if (++stage == P_STAGES) {
      stage = 0;
      phase ^= 1u;
    }
  }
  return true;
}

template <bool BF16, bool A_MN, bool B_MN>
__device__ __forceinline__ bool mma_tile_pair_n(int ncols, uint8_t* smem, uint64_t* full_bar, uint64_t* empty_bar,
                                                uint32_t peer_empty, int nkb, uint32_t d_tmem, int& stage,
                                                uint32_t& phase, volatile int* abort_flag, uint64_t tlimit) {
  switch (ncols) {
    case 64:
      return mma_tile_pair<BF16, A_MN, B_MN, 64>(smem, full_bar, empty_bar, peer_empty, nkb, d_tmem, stage, phase,
                                                 abort_flag, tlimit);
    case 128:
      return mma_tile_pair<BF16, A_MN, B_MN, 128>(smem, full_bar, empty_bar, peer_empty, nkb, d_tmem, stage, phase,
                                                  abort_flag, tlimit);
    case 192:
      return mma_tile_pair<BF16, A_MN, B_MN, 192>(smem, full_bar, empty_bar, peer_empty, nkb, d_tmem, stage, phase,
                                                  abort_flag, tlimit);
    default:
      return mma_tile_pair<BF16, A_MN, B_MN, 256>(smem, full_bar, empty_bar, peer_empty, nkb, d_tmem, stage, phase,
                                                  abort_flag, tlimit);
  }
}

// 32 x 32 fp32 transpose within a warp: lane l passes its 32 values (column l of the
// block) and receives row l (32 values).
__device__ __forceinline__ void warp_transpose32(float* stage, float* v, int lane) {
  constexpr int P = P_XPOSE_PITCH / 4;
#pragma unroll
  for (int j = 0; j < 32; ++j) stage[j * P + lane] = v[j];
  __syncwarp();
#pragma unroll
  for (int j = 0; j < 32; ++j) v[j] = stage[lane * P + j];
  __syncwarp();
}

template <bool BF16>
__global__ void __launch_bounds__(P_THREADS, 1)
    lmce_bwd_pair_kernel(const __grid_constant__ CUtensorMap map_wk, const __grid_constant__ CUtensorMap map_wmn,
                         const __grid_constant__ CUtensorMap map_xk, const __grid_constant__ CUtensorMap map_xmn,
                         const __grid_constant__ CUtensorMap map_gk, const __grid_constant__ CUtensorMap map_gmn,
                         const BwdParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + P_STAGES * P_STAGE_BYTES);
  uint64_t* empty_bar = full_bar + P_STAGES;
  uint64_t* tfull_bar = empty_bar + P_STAGES;
  uint64_t* tempty_bar = tfull_bar + 2;
  uint64_t* drain_bar = tempty_bar + 2;
  uint64_t* sched_full = drain_bar + 1;
  uint64_t* sched_empty = sched_full + SCHED_DEPTH;  // barriers end below byte 256 of the block
  // 16-byte aligned ring: the leader writes the peer's entries with one v4 cluster store
  BwdTile* ring = reinterpret_cast<BwdTile*>(smem + P_STAGES * P_STAGE_BYTES + 256);
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(ring + SCHED_DEPTH);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = __shfl_sync(0xffffffffu, threadIdx.x / 32, 0);
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();  // 0 = leader
  // per-warp epilogue staging (after the 1 KB barrier block), then the GT tiles' row data
  uint8_t* xstage = smem + P_STAGES * P_STAGE_BYTES + 1024 + (warp >= 2 ? warp - 2 : 0) * 32 * P_XPOSE_PITCH;
  float* row_lse = reinterpret_cast<float*>(smem + P_STAGES * P_STAGE_BYTES + 1024 + P_XPOSE_BYTES);
  int* row_lbl = reinterpret_cast<int*>(row_lse + P_RB);
  const PairGeom geo = make_pair_geom(p);
  int* ticket = p.sync;
  int* gdone = p.sync + 1;
  int* consumed = p.sync + 1 + p.n_chunks;
  int* dxchain = p.sync + 1 + 2 * p.n_chunks;
  int* xdone = dxchain + (p.rows_pad / BM) * geo.nh;

  if (threadIdx.x == 0) {
    for (int s = 0; s < P_STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull_bar[b], 1);
      mbar_init(&tempty_bar[b], 2 * P_EPI);
    }
    mbar_init(drain_bar, 1);
    for (int s = 0; s < SCHED_DEPTH; ++s) {
      mbar_init(&sched_full[s], 1);
      // leader's: its UMMA lane and epilogue, the peer's producer and epilogue
      mbar_init(&sched_empty[s], 2 + 2 * P_EPI);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&map_wk);
    tma_prefetch_desc(&map_wmn);
    tma_prefetch_desc(&map_xk);
    tma_prefetch_desc(&map_xmn);
    tma_prefetch_desc(&map_gk);
    tma_prefetch_desc(&map_gmn);
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_holder, TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // the peer's barriers exist before any remote arrive or copy
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  const uint64_t tlimit = p.timeout_ns;
  const uint32_t leader_sched_empty = mapa_shared(smem_u32(sched_empty), 0);

  if (warp == 0) {
    // ------------------------------------------- scheduler + TMA producer ---
    if (lane == 0) {
      int stage = 0, slot = 0;
      uint32_t phase = 0, sphase = 0;
      int issued = 0;
      bool ok = true;
      PairCursor cur;
      cur.init();
      int g_ready_chunk = -1, gbuf_free_chunk = -1;
      int next_ticket = rank == 0 ? atomicAdd(ticket, 1) : 0;
      const uint32_t full_leader = mapa_shared(smem_u32(full_bar), 0);
      const uint32_t peer_ring = mapa_shared(smem_u32(ring), 1);
      const uint32_t peer_sched_full = mapa_shared(smem_u32(sched_full), 1);
      for (;;) {
        BwdTile t;
        if (rank == 0) {
          if (!mbar_wait_cluster(&sched_empty[slot], sphase ^ 1u, abort_flag, tlimit)) {
            ok = false;
            break;
          }
          const bool has = cur.decode(geo, next_ticket, t);
          if (!has) t.kind = BK_END;
          // dependencies (before the tile is handed out, so both CTAs load after them)
          bool acquired = false;
          if (t.kind == BK_G) {
            if (t.chunk >= NUM_GBUF && t.chunk > gbuf_free_chunk) {
              const int prev = t.chunk - NUM_GBUF;
              ok = wait_counter(&consumed[prev], 2 * (geo.nDX() + geo.nDW(prev)), abort_flag, tlimit);
              if (ok) gbuf_free_chunk = t.chunk;
            }
          } else if ((t.kind == BK_DX || t.kind == BK_DW) && t.chunk > g_ready_chunk) {
            ok = wait_counter(&gdone[t.chunk], 2 * geo.nG(t.chunk), abort_flag, tlimit);
            if (ok) g_ready_chunk = t.chunk;
            acquired = true;
          }
          if (!ok) break;
          if (acquired) asm volatile("fence.proxy.async.global;" ::: "memory");
          {
            volatile int* e = reinterpret_cast<volatile int*>(&ring[slot]);
            e[0] = t.kind;
            e[1] = t.chunk;
            e[2] = t.m;
            e[3] = t.n;
          }
          st_shared_cluster_v4(peer_ring + slot * sizeof(BwdTile), t.kind, t.chunk, t.m, t.n);
          mbar_arrive(&sched_full[slot]);
          mbar_arrive_cluster(peer_sched_full + 8u * slot);
          if (++slot == SCHED_DEPTH) {
            slot = 0;
            sphase ^= 1u;
          }
          if (!has) break;
          next_ticket = atomicAdd(ticket, 1);
        } else {
          if (!mbar_wait_cluster(&sched_full[slot], sphase, abort_flag, tlimit)) {
            ok = false;
            break;
          }
          t = read_ring(&ring[slot]);
          mbar_arrive_cluster(leader_sched_empty + 8u * slot);
          if (++slot == SCHED_DEPTH) {
            slot = 0;
            sphase ^= 1u;
          }
          if (t.kind == BK_END) break;
          // G was written by other CTAs' generic stores and acquired by the leader
          if (t.kind == BK_DX || t.kind == BK_DW) asm volatile("fence.proxy.async.global;" ::: "memory");
        }

        const int nkb = geo.num_kb(t, p.H);
        const int gbuf = t.chunk % NUM_GBUF;
        const int r = static_cast<int>(rank);
        const int half_n = t.kind == BK_DW ? BM : geo.rows_n(t.m) / 2;  // this CTA's share of N
        for (int kb = 0; kb < nkb; ++kb) {
          if (!mbar_wait(&empty_bar[stage], phase ^ 1u, abort_flag, tlimit)) {
            ok = false;
            break;
          }
          uint8_t* sa = smem + stage * P_STAGE_BYTES;
          uint8_t* sb = sa + P_A_BYTES;
          if (rank == 0) mbar_arrive_expect_tx(&full_bar[stage], 2 * P_STAGE_BYTES);
          const uint32_t fb = full_leader + 8u * stage;
          const int k0 = kb * BK;
          if (t.kind == BK_G) {
            tma_load_2d_pair(sa, &map_wk, fb, k0, t.chunk * p.v_chunk + t.n * P_RB + BM * r);
            tma_load_2d_pair(sb, &map_xk, fb, k0, t.m * P_RB + half_n * r);
          } else if (t.kind == BK_DX) {
            tma_load_3d_pair(sa, &map_wmn, fb, 0, t.chunk * p.v_chunk + k0, (t.n * BN + BM * r) / 64);
            tma_load_2d_pair(sb, &map_gk, fb, k0, gbuf * p.rows_pad + t.m * P_RB + half_n * r);
          } else {
            tma_load_3d_pair(sa, &map_gmn, fb, 0, gbuf * p.rows_pad + k0, (t.m * P_RB + BM * r) / 64);
            tma_load_3d_pair(sb, &map_xmn, fb, 0, k0, (t.n * BN + BM * r) / 64);
          }
          ++issued;
          if (++stage == P_STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
      }
      if (!ok) {
        raise_error(p.err, ERR_TIMEOUT);
        *abort_flag = 1;
        if (rank == 0) {
          const int outstanding = issued < P_STAGES ? issued : P_STAGES;
          for (int i = 1; i <= outstanding; ++i) {
            int s = stage - i;
            uint32_t ph = phase;
            if (s < 0) {
              s += P_STAGES;
              ph ^= 1u;
            }
            volatile int no_abort = 0;
            mbar_wait(&full_bar[s], ph, &no_abort, tlimit);
          }
        }
      }
    }
  } else if (warp == 1) {
    // -------------------------------------------------- UMMA issuer (leader) ---
    if (lane == 0 && rank == 0) {
      const uint32_t peer_empty = mapa_shared(smem_u32(empty_bar), 1);
      const uint32_t peer_tfull = mapa_shared(smem_u32(tfull_bar), 1);
      int stage = 0, slot = 0, acc = 0;
      uint32_t phase = 0, sphase = 0, acc_phase = 0;
      bool ok = true;
      for (;;) {
        if (!mbar_wait(&sched_full[slot], sphase, abort_flag, tlimit)) {
          ok = false;
          break;
        }
        const BwdTile t = read_ring(&ring[slot]);
        mbar_arrive(&sched_empty[slot]);
        if (++slot == SCHED_DEPTH) {
          slot = 0;
          sphase ^= 1u;
        }
        if (t.kind == BK_END) break;
        if (!mbar_wait_cluster(&tempty_bar[acc], acc_phase ^ 1u, abort_flag, tlimit)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
        const int nkb = geo.num_kb(t, p.H);
        if (t.kind == BK_G)
          ok = mma_tile_pair_n<BF16, false, false>(geo.rows_n(t.m), smem, full_bar, empty_bar, peer_empty, nkb,
                                                   d_tmem, stage, phase, abort_flag, tlimit);
        else if (t.kind == BK_DX)
          ok = mma_tile_pair_n<BF16, true, false>(geo.rows_n(t.m), smem, full_bar, empty_bar, peer_empty, nkb,
                                                  d_tmem, stage, phase, abort_flag, tlimit);
        else if (t.kind == BK_DW)
          ok = mma_tile_pair<BF16, true, true, BN>(smem, full_bar, empty_bar, peer_empty, nkb, d_tmem, stage, phase,
                                                   abort_flag, tlimit);
        if (!ok) break;
        umma_commit_pair(smem_u32(&tfull_bar[acc]));  // also fires when no UMMA was issued
        umma_commit_pair(peer_tfull + 8u * acc);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
      if (!ok) {
        raise_error(p.err, ERR_TIMEOUT);
        *abort_flag = 1;
      }
      umma_commit_pair(smem_u32(drain_bar));
      volatile int no_abort = 0;
      mbar_wait(drain_bar, 0, &no_abort, tlimit);
    }
  } else {
    // ---------------------------------------------------------- epilogue ---
    const int q = warp & 3;      // TMEM lane quadrant
    const int ch = (warp - 2) >> 2;  // column half of each tile this warp handles
    const int et = static_cast<int>(threadIdx.x) - EPI_THREAD0;
    const int lrow = BM * static_cast<int>(rank) + q * 32 + lane;  // this thread's M index within the 256
    const uint32_t lane_base = static_cast<uint32_t>(q * 32) << 16;
    const uint32_t leader_tempty = mapa_shared(smem_u32(tempty_bar), 0);
    const float gl = p.grad_loss ? *p.grad_loss : 1.0f;
    const float dscale = gl / (*p.denom) / p.gscale;
    int slot = 0, acc = 0;
    uint32_t sphase = 0, acc_phase = 0;
    bool ok = true;
    for (;;) {
      if (!mbar_wait_cluster(&sched_full[slot], sphase, abort_flag, tlimit)) {
        ok = false;
        break;
      }
      const BwdTile t = read_ring(&ring[slot]);
      mbar_arrive_cluster(leader_sched_empty + 8u * slot);
      if (++slot == SCHED_DEPTH) {
        slot = 0;
        sphase ^= 1u;
      }
      if (t.kind == BK_END) break;
      if (t.kind == BK_XCH) {
        if (!mbar_wait(&tfull_bar[acc], acc_phase, abort_flag, tlimit)) {
          ok = false;
          break;
        }
        // this CTA sums rows [128 * rank, 128 * rank + 128) of the 256-row block (the first
        // four epilogue warps, on their own named barrier)
        if (ch == 0)
          exchange_rows_range<BF16, 2>(p, t.m * P_RB + BM * static_cast<int>(rank), geo.n_lab, geo.nh * 2, t,
                                       xdone, 2 * geo.nX, abort_flag, tlimit);
        mbar_arrive_cluster(leader_tempty + 8u * acc);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1u;
        }
        continue;
      }
      const bool have_acc = geo.num_kb(t, p.H) > 0;
      const int w = geo.width(t.chunk);
      const int ncols = t.kind == BK_DW ? BN : geo.rows_n(t.m);
      const int row_blk0 = t.m * P_RB;  // first token row of a GT / DXT tile

      if (t.kind == BK_G) {
        // row data of the tile's 256 rows, loaded while the UMMAs still run: lse * log2(e)
        // (+inf for rows past the labelled ones, so their probabilities are 0) and the label
        // relative to the chunk (-1: none). The previous GT tile's readers are past the
        // barrier of its publish step.
        for (int r = et; r < P_RB; r += P_EPI) {
          const int row = row_blk0 + r;
          const bool ok_r = row < geo.n_lab;
          row_lse[r] = ok_r ? p.lse_lab[row] * LOG2E : INFINITY;
          const int y = ok_r ? p.lbl_lab[row] : -1;
          row_lbl[r] = y >= 0 ? y - t.chunk * p.v_chunk : -1;
        }
        named_bar<1, P_EPI>();
      }
      if (t.kind == BK_DX && t.chunk > 0) {
        // dX^T columns of this tile were last written by DXT(chunk - 1) on some pair
        if (et == 0 && !wait_counter(&dxchain[t.m * geo.nh + t.n], 2 * t.chunk, abort_flag, tlimit)) {
          raise_error(p.err, ERR_TIMEOUT);
          *abort_flag = 1;
        }
        named_bar<1, P_EPI>();
      }
      if (!mbar_wait(&tfull_bar[acc], acc_phase, abort_flag, tlimit)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t taddr = tmem_base + lane_base + static_cast<uint32_t>(acc * BN);

#pragma unroll 1
      for (int c = ch * (ncols / 64); c < (ch + 1) * (ncols / 64); ++c) {
        uint32_t raw[32];
        float v[32];
        __syncwarp();
        tmem_ld_32x32b_x32(taddr + c * 32, raw);
        tmem_ld_wait(raw);
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = have_acc ? __uint_as_float(raw[j]) : 0.0f;

        if (t.kind == BK_G) {
          // this thread: vocab row vloc of the chunk; columns: token rows row_blk0 + c * 32 + j,
          // whose lse comes from the tile's row data (four rows per shared-memory load). The
          // one-hot term is checked only when a label of the 32 rows falls in this warp's 32
          // vocab rows (a ballot; rare for wide vocab chunks).
          const int vloc = t.n * P_RB + lrow;
          const int vbase = vloc - lane;
          const float* lse_s = row_lse + c * 32;
          const int y_l = row_lbl[c * 32 + lane];
          const bool hit = __ballot_sync(0xffffffffu, y_l >= vbase && y_l < vbase + 32) != 0u;
          const float gs = vloc < w ? p.gscale : 0.0f;
          uint16_t* st16 = reinterpret_cast<uint16_t*>(xstage);
#pragma unroll
          for (int j4 = 0; j4 < 8; ++j4) {
            const float4 L = reinterpret_cast<const float4*>(lse_s)[j4];
            const float lj[4] = {L.x, L.y, L.z, L.w};
            float g4[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              const int j = 4 * j4 + u;
              float pr = ex2_approx(fmaf(round_to_input<BF16>(v[j]), LOG2E, -lj[u]));
              if (hit) {  // warp-uniform
                if (__shfl_sync(0xffffffffu, y_l, j) == vloc) pr -= 1.0f;
              }
              g4[u] = pr * gs;
            }
            // staging rows 4 * j4 .. + 3 (tokens), column lane (vocab); one conversion per two values
#pragma unroll
            for (int u = 0; u < 4; u += 2) {
              const uint32_t two = pack2<BF16>(g4[u], g4[u + 1]);
              st16[(4 * j4 + u) * (ROW_STAGE_PITCH / 2) + lane] = static_cast<uint16_t>(two & 0xffffu);
              st16[(4 * j4 + u + 1) * (ROW_STAGE_PITCH / 2) + lane] = static_cast<uint16_t>(two >> 16);
            }
          }
          __syncwarp();
          // copy out: 8 token rows x 64 bytes (32 vocab columns) per instruction
          char* gbase = reinterpret_cast<char*>(p.g) +
                        (static_cast<size_t>(t.chunk % NUM_GBUF) * p.rows_pad * p.v_chunk + t.n * P_RB +
                         BM * static_cast<int>(rank) + q * 32) * 2;
#pragma unroll
          for (int i2 = 0; i2 < 4; ++i2) {
            const int rr = i2 * 8 + (lane >> 2);
            const int piece = lane & 3;
            const uint4 u = *reinterpret_cast<const uint4*>(xstage + rr * ROW_STAGE_PITCH + piece * 16);
            *reinterpret_cast<uint4*>(gbase + static_cast<size_t>(row_blk0 + c * 32 + rr) * p.v_chunk * 2 +
                                      piece * 16) = u;
          }
          __syncwarp();
        } else if (t.kind == BK_DX) {
          // this thread: hidden index h; columns: token rows (compacted) row_blk0 + c * 32 + j
          const int h = t.n * BN + lrow;
          if (h < p.H) {
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] *= dscale;
            float* accp = p.dx_acc + static_cast<size_t>(h) * p.rows_pad + row_blk0 + c * 32;
            if (t.chunk > 0) {
#pragma unroll
              for (int j = 0; j < 32; j += 4) {
                const float4 a4 = __ldcg(reinterpret_cast<const float4*>(accp + j));
                v[j] += a4.x;
                v[j + 1] += a4.y;
                v[j + 2] += a4.z;
                v[j + 3] += a4.w;
              }
            }
            if (t.chunk + 1 < geo.C) {
#pragma unroll
              for (int j = 0; j < 32; j += 4)
                __stcg(reinterpret_cast<float4*>(accp + j), make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]));
            }
          }
          if (t.chunk + 1 == geo.C) {
            // transpose: lane l gets token row row_blk0 + c * 32 + l, hidden h0 .. h0 + 31
            warp_transpose32(reinterpret_cast<float*>(xstage), v, lane);
            const int h0 = t.n * BN + BM * static_cast<int>(rank) + q * 32;
            const int row = row_blk0 + c * 32 + lane;
            if (h0 < p.H && row < geo.n_lab) {
              const size_t trow = static_cast<size_t>(p.row_idx[row]);
              if (p.dx_out_f32 != nullptr) {
                float* dst = p.dx_out_f32 + trow * p.H + h0;
#pragma unroll
                for (int j = 0; j < 32; j += 4)
                  *reinterpret_cast<float4*>(dst + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
              }
              if (p.dx_out != nullptr)
                store32_dtype<BF16>(reinterpret_cast<char*>(p.dx_out) + (trow * p.H + h0) * 2, v);
            }
          }
        } else {  // BK_DW: this thread: vocab row of the chunk; columns: hidden h0 + j
          const int h0 = t.n * BN + c * 32;
          if (h0 < p.H) {
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] *= dscale;
            const int v0 = t.m * P_RB + BM * static_cast<int>(rank) + q * 32;  // warp's first vocab row
            char* dbase = reinterpret_cast<char*>(p.dw_out) +
                          ((static_cast<size_t>(t.chunk) * p.v_chunk + v0) * p.H + h0) * 2;
            store_rows32<BF16>(xstage, v, dbase, static_cast<size_t>(p.H) * 2, 0, lane,
                               [v0, w](int rr) { return v0 + rr < w; });
          }
        }
      }
      tc_fence_before();
      mbar_arrive_cluster(leader_tempty + 8u * acc);
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1u;
      }
      // publish this CTA's half of the tile
      named_bar<1, P_EPI>();  // all of this CTA's stores of the tile happen before its count
      if (t.kind == BK_G) {
        if (et == 0) {
          __threadfence();
          atomicAdd(&gdone[t.chunk], 1);
        }
      } else if (t.kind == BK_DX) {
        if (et == 0) {
          const bool x_last = geo.xch && t.chunk + 1 == geo.C;
          if (x_last)
            __threadfence_system();
          else
            __threadfence();
          atomicAdd(&dxchain[t.m * geo.nh + t.n], 1);
          atomicAdd(&consumed[t.chunk], 1);
          if (x_last)
            multimem_st_release_b32(p.x_flags_mc + p.x_world +
                                        ((static_cast<size_t>(t.m) * p.x_world + p.x_rank) * geo.nh + t.n) * 2 + rank,
                                    p.x_epoch);
        }
      } else if (et == 0) {
        __threadfence();
        atomicAdd(&consumed[t.chunk], 1);
      }
    }
    if (!ok) {
      raise_error(p.err, ERR_TIMEOUT);
      *abort_flag = 1;
    }
    if (geo.xch && blockIdx.x == 0) {
      if (et == 0 && geo.nX == 0) multimem_st_release_b32(p.x_flags_mc + p.x_rank, p.x_epoch);
      for (int r = et; r < p.x_world; r += P_EPI) {
        if (!*abort_flag && !wait_flag_sys(p.x_flags + r, p.x_epoch, abort_flag, tlimit)) {
          raise_error(p.err, ERR_TIMEOUT);
          *abort_flag = 1;
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync();  // the leader's UMMAs into the peer's TMEM have drained
  tc_fence_after();
  if (warp == 1) {
    __syncwarp();
    tmem_dealloc_pair(tmem_base, TMEM_COLS);
  }
}

}  // namespace lmce
