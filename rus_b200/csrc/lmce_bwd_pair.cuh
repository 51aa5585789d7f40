// Persistent backward of the lm_head CE head on CTA pairs (tcgen05 cta_group::2).
//
// Same work as lmce_bwd_kernel (recomputed logits -> G, dX and dW GEMMs), laid out
// so that the two CTAs of a cluster share every tile: the MMA is 256 x N, each CTA
// stages its 128 rows of A and N/2 rows of B. A stage holds K = 128 (64 KB per CTA,
// three stages), and each operand of a stage arrives as one TMA box that reads 256
// contiguous bytes of each of its 128 rows, which keeps the pair UMMA fed (about 63
// bytes per clock per SM, where 128-byte rows give 46-52). The token rows are the N
// dimension of the tiles that contract over them, so a row block's tile is 128 or 256 tokens wide
// (padded to 128, not to the M tile). The gradient tile is stored transposed, as
// G^T [vocab][token] (the TMEM layout: each epilogue thread holds one vocab row), so
// the epilogue writes it without a shared-memory transpose; the dX GEMM reads it as an
// MN-major B operand and the dW GEMM as a K-major A operand.
//   GT(c)   vocab block jv (M, 256) x row block i (N = 128 or 256) of G^T = W_c . X_lab^T,
//           K = H: the epilogue forms G = (softmax - onehot) * 2^15 in the input dtype
//           (the prescale folded into the exponent) and writes rows of G^T to G buffer
//           c % NUM_GBUF (replaces the reference's pass-2 GEMM + lm_head_piece_kernel
//           MODE 1, solution/ops.py:287-319, solution/kernels.py:517-531)
//   DXT(c)  hidden block p (M) x row block i (N) of dX^T += W_c^T . G_c^T, K = chunk
//           width; fp32 accumulation in a [H][rows] buffer in chunk order: TMA stores
//           (chunk 0) and TMA adds (later chunks) of 32 x 32 boxes; the last chunk reads
//           the sum back, adds its own, scales by grad_loss / denom / 2^15, transposes
//           through shared memory and scatters rows to token order (replaces ops.py:320
//           and 337-338)
//   DW(c)   vocab block jv (M) x hidden block p (N = 256) of dW = G_c^T . X_lab, K =
//           labelled tokens (new: the reference returns None for the weight, ops.py:339)
// The tile list, its order, the dependency counters and the fused cross-GPU exchange
// follow lmce_bwd_kernel; every count covers both CTAs of a pair: each epilogue warp
// publishes its rows of a GT tile (no CTA barrier: 16 counts per tile), each CTA its half
// of a DXT tile, and a tile that read a G buffer releases it when its accumulator is full
// (its UMMAs have read their operands by then). The pair leader (cluster rank 0) claims
// tickets, checks dependencies and hands each tile to both CTAs' schedule rings (the
// peer's through distributed shared memory); only the leader issues UMMAs. Every wait is
// bounded.
#pragma once

#include "lmce_bwd.cuh"
#include "lmce_prof.cuh"

namespace lmce {

// A stage holds K = 128 of both operands (two 64-element swizzle blocks), and every
// operand arrives as one 3-D TMA box {64, 128, 2} that reads 256 contiguous bytes of
// each of its 128 rows: measured on B200 at ~63 bytes per clock per SM against ~46 for
// two 2-D {64, 128} boxes (128 bytes per row), while a 256 x 256 pair UMMA consumes 64.
constexpr int P_KB = 2 * BK;     // K per stage
constexpr int P_STAGES = 3;
constexpr int P_THREADS = 320;  // warp 0 producer, warp 1 UMMA, warps 2-9 epilogue (two per TMEM lane quadrant)
constexpr int P_EPI = 256;
constexpr int P_EPI_WARPS = P_EPI / 32;
constexpr int P_A_BYTES = BM * P_KB * 2;                   // 128 rows x 128 k: 32 KB
constexpr int P_B_BYTES = BM * P_KB * 2;                   // up to 128 rows (N / 2) x 128 k: 32 KB
constexpr int P_STAGE_BYTES = P_A_BYTES + P_B_BYTES;       // 64 KB
constexpr int P_RB = 256;                                  // token rows per row block
// One epilogue warp's staging slice: a 32 x 32 fp32 block in the 128-byte swizzled layout
// of a TMA box (4 KB, 1024-byte aligned), also used for 16-bit row staging and transposes.
constexpr int P_SLICE_BYTES = 32 * 32 * 4;
constexpr int P_XPOSE_PITCH = 17;                          // fp32 32 x 32 transpose in two halves, in floats
constexpr int P_XPOSE_BYTES = 8 * P_SLICE_BYTES;           // slices of the eight epilogue warps
// A GT tile's per-row data (exponent offset and chunk-local label) for the 128 token
// columns a warp handles, kept in the warp's slice behind its 16-bit row staging.
constexpr int P_ROWDATA_OFF = 32 * ROW_STAGE_PITCH;        // 2560
static_assert(P_ROWDATA_OFF + 128 * 8 <= P_SLICE_BYTES, "row data fits behind the row staging");
// stages, 1 KB of barriers and ring, the staging slices, and 1 KB of slack for the
// 1024-byte alignment of the dynamic shared memory base
constexpr int PBWD_SMEM_BYTES = P_STAGES * P_STAGE_BYTES + 2048 + P_XPOSE_BYTES;
static_assert((2 * P_STAGES + 5 + 2 * SCHED_DEPTH) * 8 <= 256, "pair barriers end below the ring");
static_assert(32 * P_XPOSE_PITCH * 4 <= P_SLICE_BYTES, "half-transpose staging fits a warp's slice");
static_assert(32 * ROW_STAGE_PITCH <= P_SLICE_BYTES, "16-bit row staging fits a warp's slice");
static_assert((P_STAGES * P_STAGE_BYTES + 1024) % 1024 == 0, "staging slices are 1024-byte aligned (128-byte swizzle)");
static_assert(PBWD_SMEM_BYTES <= 227 * 1024, "dynamic shared memory of one CTA");

struct PairGeom {
  int n_lab, nrb, nh, C, vc, V, nX;
  bool dx, dw, xch;
  __device__ __forceinline__ int width(int c) const { return min(vc, V - c * vc); }
  __device__ __forceinline__ int nvb(int c) const { return (width(c) + 255) / 256; }
  __device__ __forceinline__ int nG(int c) const { return nvb(c) * nrb; }
  __device__ __forceinline__ int nDX() const { return dx ? nh * nrb : 0; }
  __device__ __forceinline__ int nDW(int c) const { return dw ? nvb(c) * nh : 0; }
  // N of a row-block tile: 128 when at most 128 rows of the block hold labelled tokens,
  // else 256 (each CTA's half of an MN-major G^T operand is then one or two whole
  // 64-token swizzle blocks)
  __device__ __forceinline__ int rows_n(int i) const { return n_lab - i * P_RB > BM ? P_RB : BM; }
  // stages (K = 128 each) of a tile; a stage past the end of K reads zeros (TMA fill)
  __device__ __forceinline__ int num_kb(const BwdTile& t, int H) const {
    if (t.kind == BK_XCH) return 0;
    if (t.kind == BK_G) return (H + P_KB - 1) / P_KB;
    if (t.kind == BK_DX) return (width(t.chunk) + P_KB - 1) / P_KB;
    return (n_lab + P_KB - 1) / P_KB;
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
                                              uint32_t& phase, volatile int* abort_flag, uint64_t tlimit,
                                              long long& full_wait) {
  constexpr uint32_t idesc = make_idesc_f16(BF16, A_MN, B_MN, 2 * BM, NCOLS);
  for (int kb = 0; kb < nkb; ++kb) {
    LMCE_PROF(const long long t0 = clock64();)
    if (!mbar_wait(&full_bar[stage], phase, abort_flag, tlimit)) return false;
    LMCE_PROF(full_wait += clock64() - t0;)
    tc_fence_after();
    const uint32_t sa = smem_u32(smem + stage * P_STAGE_BYTES);
#pragma unroll
    for (int k = 0; k < P_KB / UMMA_K; ++k)
      umma_f16_ss_pair(d_tmem, pair_operand_desc(sa, A_MN, k), pair_operand_desc(sa + P_A_BYTES, B_MN, k), idesc,
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
                                                uint32_t& phase, volatile int* abort_flag, uint64_t tlimit,
                                                long long& full_wait) {
  switch (ncols) {
    case 128:
      return mma_tile_pair<BF16, A_MN, B_MN, 128>(smem, full_bar, empty_bar, peer_empty, nkb, d_tmem, stage, phase,
                                                  abort_flag, tlimit, full_wait);
    default:
      return mma_tile_pair<BF16, A_MN, B_MN, 256>(smem, full_bar, empty_bar, peer_empty, nkb, d_tmem, stage, phase,
                                                  abort_flag, tlimit, full_wait);
  }
}

// 32 x 32 fp32 transpose within a warp: lane l passes its 32 values (column l of the
// block) and receives row l (32 values), in two passes through a 32 x 17 staging block:
// lanes 16h .. 16h + 15 store theirs, then every lane reads its row's 16 values of them.
__device__ __forceinline__ void warp_transpose32(float* stage, float* v, int lane) {
  constexpr int P = P_XPOSE_PITCH;
  float out[32];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    if ((lane >> 4) == h) {
#pragma unroll
      for (int j = 0; j < 32; ++j) stage[j * P + (lane & 15)] = v[j];
    }
    __syncwarp();
#pragma unroll
    for (int i = 0; i < 16; ++i) out[16 * h + i] = stage[lane * P + i];
    __syncwarp();
  }
#pragma unroll
  for (int j = 0; j < 32; ++j) v[j] = out[j];
}

template <bool BF16>
__global__ void __launch_bounds__(P_THREADS, 1)
    lmce_bwd_pair_kernel(const __grid_constant__ CUtensorMap map_w, const __grid_constant__ CUtensorMap map_x,
                         const __grid_constant__ CUtensorMap map_g, const __grid_constant__ CUtensorMap map_dx,
                         const __grid_constant__ CUtensorMap map_dw, const BwdParams p) {
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
  uint8_t* xstage = smem + P_STAGES * P_STAGE_BYTES + 1024 + (warp >= 2 ? warp - 2 : 0) * P_SLICE_BYTES;
  float* row_lse = reinterpret_cast<float*>(xstage + P_ROWDATA_OFF);  // this warp's 128 token columns
  int* row_lbl = reinterpret_cast<int*>(row_lse + 128);
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
    tma_prefetch_desc(&map_w);
    tma_prefetch_desc(&map_x);
    tma_prefetch_desc(&map_g);
    tma_prefetch_desc(&map_dx);
    if (p.want_dw) tma_prefetch_desc(&map_dw);
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
  LMCE_PROF(const long long prof_t_begin = clock64();)

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
      LMCE_PROF(long long pc_sched = 0, pc_dep_g = 0, pc_dep_gd = 0, pc_empty = 0, pc_tiles = 0;)
      for (;;) {
        BwdTile t;
        LMCE_PROF(long long pt0 = clock64();)
        if (rank == 0) {
          if (!mbar_wait_cluster(&sched_empty[slot], sphase ^ 1u, abort_flag, tlimit)) {
            ok = false;
            break;
          }
          LMCE_PROF(pc_sched += clock64() - pt0; pt0 = clock64();)
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
            LMCE_PROF(pc_dep_g += clock64() - pt0;)
          } else if ((t.kind == BK_DX || t.kind == BK_DW) && t.chunk > g_ready_chunk) {
            ok = wait_counter(&gdone[t.chunk], 2 * P_EPI_WARPS * geo.nG(t.chunk), abort_flag, tlimit);
            if (ok) g_ready_chunk = t.chunk;
            acquired = true;
            LMCE_PROF(pc_dep_gd += clock64() - pt0;)
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
          LMCE_PROF(pc_sched += clock64() - pt0;)
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
        LMCE_PROF(++pc_tiles;)
        for (int kb = 0; kb < nkb; ++kb) {
          LMCE_PROF(const long long pe0 = clock64();)
          if (!mbar_wait(&empty_bar[stage], phase ^ 1u, abort_flag, tlimit)) {
            ok = false;
            break;
          }
          LMCE_PROF(pc_empty += clock64() - pe0;)
          uint8_t* sa = smem + stage * P_STAGE_BYTES;
          uint8_t* sb = sa + P_A_BYTES;
          if (rank == 0) mbar_arrive_expect_tx(&full_bar[stage], 2 * P_STAGE_BYTES);
          const uint32_t fb = full_leader + 8u * stage;
          // every operand: one {64, 128, 2} box of a 3-D view {64 elements, rows, 64-element
          // blocks}; K-major operands take two k-blocks of 128 rows, MN-major ones 128 k-rows
          // of two MN blocks
          if (t.kind == BK_G) {
            tma_load_3d_pair(sa, &map_w, fb, 0, t.chunk * p.v_chunk + t.n * P_RB + BM * r, 2 * kb);
            tma_load_3d_pair(sb, &map_x, fb, 0, t.m * P_RB + half_n * r, 2 * kb);
          } else if (t.kind == BK_DX) {
            // B: tokens of this CTA's half as MN-major blocks of G^T (two 64-token blocks; with
            // N = 128 the UMMA reads only the first)
            tma_load_3d_pair(sa, &map_w, fb, 0, t.chunk * p.v_chunk + kb * P_KB, (t.n * BN + BM * r) / 64);
            tma_load_3d_pair(sb, &map_g, fb, 0, gbuf * p.v_chunk + kb * P_KB, (t.m * P_RB + half_n * r) / 64);
          } else {
            // A: this CTA's 128 vocab rows of G^T, K-major over the tokens
            tma_load_3d_pair(sa, &map_g, fb, 0, gbuf * p.v_chunk + t.m * P_RB + BM * r, 2 * kb);
            tma_load_3d_pair(sb, &map_x, fb, 0, kb * P_KB, (t.n * BN + BM * r) / 64);
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
      LMCE_PROF(prof_store(PS_P_SCHED, pc_sched); prof_store(PS_P_DEP_G, pc_dep_g);
                prof_store(PS_P_DEP_GD, pc_dep_gd); prof_store(PS_P_EMPTY, pc_empty);
                prof_store(PS_P_TILES, pc_tiles);)
    }
  } else if (warp == 1) {
    // -------------------------------------------------- UMMA issuer (leader) ---
    if (lane == 0 && rank == 0) {
      const uint32_t peer_empty = mapa_shared(smem_u32(empty_bar), 1);
      const uint32_t peer_tfull = mapa_shared(smem_u32(tfull_bar), 1);
      int stage = 0, slot = 0, acc = 0;
      uint32_t phase = 0, sphase = 0, acc_phase = 0;
      bool ok = true;
      long long full_g = 0, full_dx = 0, full_dw = 0;
      LMCE_PROF(long long pc_msched = 0, pc_tempty = 0, kb_g = 0, kb_dx = 0, kb_dw = 0; int tl_i = 0;
                const long long pm_loop0 = clock64();)
      for (;;) {
        LMCE_PROF(long long pm0 = clock64();)
        if (!mbar_wait(&sched_full[slot], sphase, abort_flag, tlimit)) {
          ok = false;
          break;
        }
        LMCE_PROF(pc_msched += clock64() - pm0;)
        const BwdTile t = read_ring(&ring[slot]);
        mbar_arrive(&sched_empty[slot]);
        if (++slot == SCHED_DEPTH) {
          slot = 0;
          sphase ^= 1u;
        }
        if (t.kind == BK_END) break;
        LMCE_PROF(pm0 = clock64();)
        if (!mbar_wait_cluster(&tempty_bar[acc], acc_phase ^ 1u, abort_flag, tlimit)) {
          ok = false;
          break;
        }
        LMCE_PROF(pc_tempty += clock64() - pm0;
                  if (unsigned long long* e = prof_entry(tl_i++)) e[4] = global_timer_ns();)
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
        const int nkb = geo.num_kb(t, p.H);
        if (t.kind == BK_G) {
          ok = mma_tile_pair_n<BF16, false, false>(geo.rows_n(t.m), smem, full_bar, empty_bar, peer_empty, nkb,
                                                   d_tmem, stage, phase, abort_flag, tlimit, full_g);
          LMCE_PROF(kb_g += nkb;)
        } else if (t.kind == BK_DX) {
          ok = mma_tile_pair_n<BF16, true, true>(geo.rows_n(t.m), smem, full_bar, empty_bar, peer_empty, nkb,
                                                 d_tmem, stage, phase, abort_flag, tlimit, full_dx);
          LMCE_PROF(kb_dx += nkb;)
        } else if (t.kind == BK_DW) {
          ok = mma_tile_pair<BF16, false, true, BN>(smem, full_bar, empty_bar, peer_empty, nkb, d_tmem, stage, phase,
                                                    abort_flag, tlimit, full_dw);
          LMCE_PROF(kb_dw += nkb;)
        }
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
      LMCE_PROF(prof_store(PS_M_SCHED, pc_msched); prof_store(PS_M_TEMPTY, pc_tempty);
                prof_store(PS_M_FULL_G, full_g); prof_store(PS_M_FULL_DX, full_dx); prof_store(PS_M_FULL_DW, full_dw);
                prof_store(PS_M_KB_G, kb_g); prof_store(PS_M_KB_DX, kb_dx); prof_store(PS_M_KB_DW, kb_dw);
                prof_store(PS_M_LOOP, clock64() - pm_loop0);)
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
    bool dw_pending = false;  // this warp's last dW tile may still have TMA stores reading its slice
    LMCE_PROF(long long e_sched = 0, e_chain = 0, e_xch = 0, tf_g = 0, tf_dx = 0, tf_dw = 0, wk_g = 0, wk_dx = 0,
              wk_dw = 0, n_g = 0, n_dx = 0, n_dw = 0;
              int tl_i = 0; const long long pl0 = clock64(); long long pe_tile = 0; unsigned long long* tle = nullptr;)
    for (;;) {
      LMCE_PROF(long long pe0 = clock64();)
      if (!mbar_wait_cluster(&sched_full[slot], sphase, abort_flag, tlimit)) {
        ok = false;
        break;
      }
      LMCE_PROF(e_sched += clock64() - pe0;)
      const BwdTile t = read_ring(&ring[slot]);
      mbar_arrive_cluster(leader_sched_empty + 8u * slot);
      if (++slot == SCHED_DEPTH) {
        slot = 0;
        sphase ^= 1u;
      }
      if (t.kind == BK_END) break;
      if (dw_pending) {  // the last dW tile's TMA stores have left this warp's slice
        if (lane == 0) bulk_wait_read_all();
        __syncwarp();
        dw_pending = false;
      }
      LMCE_PROF(tle = et == 0 ? prof_entry(tl_i++) : nullptr;
                if (tle) { tle[0] = t.kind; tle[1] = t.chunk; tle[2] = t.m; tle[3] = t.n; tle[5] = global_timer_ns(); })
      if (t.kind == BK_XCH) {
        if (!mbar_wait(&tfull_bar[acc], acc_phase, abort_flag, tlimit)) {
          ok = false;
          break;
        }
        LMCE_PROF(pe0 = clock64(); if (tle) tle[6] = global_timer_ns();)
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
        LMCE_PROF(e_xch += clock64() - pe0; if (tle) tle[7] = global_timer_ns();)
        continue;
      }
      const bool have_acc = geo.num_kb(t, p.H) > 0;
      const int w = geo.width(t.chunk);
      const int ncols = t.kind == BK_DW ? BN : geo.rows_n(t.m);
      const int row_blk0 = t.m * P_RB;  // first token row of a GT / DXT tile
      const int c_lo = ch * (ncols / 64), c_hi = (ch + 1) * (ncols / 64);  // this warp's 32-column chunks

      if (t.kind == BK_G) {
        // row data of this warp's token columns, loaded into its slice while the UMMAs still
        // run: lse * log2(e) minus log2 of the G prescale (so the exponential yields p * 2^15
        // directly; +inf for rows past the labelled ones, so their G is 0) and the label
        // relative to the chunk (-1: none)
        for (int i = lane; i < (c_hi - c_lo) * 32; i += 32) {
          const int row = row_blk0 + c_lo * 32 + i;
          const bool ok_r = row < geo.n_lab;
          row_lse[i] = ok_r ? fmaf(p.lse_lab[row], LOG2E, -GSCALE_LOG2) : INFINITY;
          const int y = ok_r ? p.lbl_lab[row] : -1;
          row_lbl[i] = y >= 0 ? y - t.chunk * p.v_chunk : -1;
        }
        __syncwarp();
      }
      // DXT: this thread's row h_dx of the fp32 accumulator dX^T[h][rows]. Chunks before the
      // last leave their partial sums to the memory system (a TMA store for chunk 0, TMA
      // adds after it, in chunk order through dxchain). The last chunk reads the sum of the
      // others back (the first 32 columns while the UMMAs still run), adds its own and
      // writes dX in token order.
      const int h_dx = t.n * BN + lrow;
      const bool dx_last = t.kind == BK_DX && t.chunk + 1 == geo.C;
      float* acc_row = p.dx_acc + static_cast<size_t>(h_dx) * p.rows_pad + row_blk0;
      const bool dx_prev = dx_last && t.chunk > 0 && h_dx < p.H;
      float4 pre[8];
      if (t.kind == BK_DX && t.chunk > 0) {
        LMCE_PROF(pe0 = clock64();)
        // dX^T columns of this tile were last written by DXT(chunk - 1) on some pair
        if (et == 0 && !wait_counter(&dxchain[t.m * geo.nh + t.n], 2 * t.chunk, abort_flag, tlimit)) {
          raise_error(p.err, ERR_TIMEOUT);
          *abort_flag = 1;
        }
        named_bar<1, P_EPI>();
        LMCE_PROF(e_chain += clock64() - pe0;)
        if (!dx_last && lane == 0) fence_async_global();  // the acquired sum, before this warp's TMA adds
        if (dx_prev) {
#pragma unroll
          for (int j = 0; j < 8; ++j) pre[j] = __ldcg(reinterpret_cast<const float4*>(acc_row + c_lo * 32) + j);
        }
      }
      LMCE_PROF(pe0 = clock64();)
      if (!mbar_wait(&tfull_bar[acc], acc_phase, abort_flag, tlimit)) {
        ok = false;
        break;
      }
      LMCE_PROF(const long long dtf = clock64() - pe0; pe_tile = clock64();
                if (t.kind == BK_G) tf_g += dtf; else if (t.kind == BK_DX) tf_dx += dtf; else tf_dw += dtf;
                if (tle) tle[6] = global_timer_ns();)
      tc_fence_after();
      const uint32_t taddr = tmem_base + lane_base + static_cast<uint32_t>(acc * BN);
      // A DXT or dW tile releases its G buffer as soon as its accumulator is full: its UMMAs have
      // read all of their G operand by then (TMA loads that completed before they were issued),
      // so the release waits for none of the tile's stores.
      if ((t.kind == BK_DW || t.kind == BK_DX) && et == 0) atomicAdd(&consumed[t.chunk], 1);

#pragma unroll 1
      for (int c = c_lo; c < c_hi; ++c) {
        uint32_t raw[32];
        float v[32];
        __syncwarp();
        tmem_ld_32x32b_x32(taddr + c * 32, raw);
        tmem_ld_wait(raw);
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = have_acc ? __uint_as_float(raw[j]) : 0.0f;

        if (t.kind == BK_G) {
          // this thread: vocab row vloc of the chunk; columns: token rows row_blk0 + c * 32 + j,
          // whose exponent offset comes from the tile's row data (four rows per shared-memory
          // load). The one-hot term is checked only when a label of the 32 rows falls in this
          // warp's 32 vocab rows (a ballot; rare for wide vocab chunks). The warp's 32 rows of
          // G^T (64 bytes each) go out through its staging slice, 8 rows x 64 bytes per store.
          const int vloc = t.n * P_RB + lrow;
          const int vbase = vloc - lane;
          const float* lse_s = row_lse + (c - c_lo) * 32;
          const int y_l = row_lbl[(c - c_lo) * 32 + lane];
          const bool hit = __ballot_sync(0xffffffffu, y_l >= vbase && y_l < vbase + 32) != 0u;
          const bool in_chunk = vloc < w;  // rows past the chunk's last vocab row store zeros
#pragma unroll
          for (int j4 = 0; j4 < 8; ++j4) {
            const float4 L = reinterpret_cast<const float4*>(lse_s)[j4];
            const float lj[4] = {L.x, L.y, L.z, L.w};
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              const int j = 4 * j4 + u;
              float pr = ex2_approx(fmaf(round_to_input<BF16>(v[j]), LOG2E, -lj[u]));  // p * 2^15
              if (hit) {  // warp-uniform
                if (__shfl_sync(0xffffffffu, y_l, j) == vloc) pr -= GSCALE;
              }
              v[j] = in_chunk ? pr : 0.0f;
            }
          }
          char* gbase = reinterpret_cast<char*>(p.g) +
                        ((static_cast<size_t>(t.chunk % NUM_GBUF) * p.v_chunk + vbase) * p.rows_pad + row_blk0 +
                         c * 32) * 2;
          store_rows32<BF16>(xstage, v, gbase, static_cast<size_t>(p.rows_pad) * 2, 0, lane,
                             [](int) { return true; });
        } else if (t.kind == BK_DX && !dx_last) {
          // this warp's 32 hidden rows x 32 token columns, scaled, into its slice in the 128-byte
          // swizzled box layout (16-byte piece i of row r at position i ^ (r % 8): conflict-free),
          // then one TMA store / add of the box into dX^T
          float4* sl = reinterpret_cast<float4*>(xstage);
          if (c > c_lo && lane == 0) bulk_wait_read_all();  // the previous chunk's box has left the slice
          __syncwarp();
#pragma unroll
          for (int i = 0; i < 8; ++i)
            sl[lane * 8 + (i ^ (lane & 7))] =
                make_float4(v[4 * i] * dscale, v[4 * i + 1] * dscale, v[4 * i + 2] * dscale, v[4 * i + 3] * dscale);
          fence_async_shared();
          __syncwarp();
          const int by = t.n * BN + BM * static_cast<int>(rank) + q * 32;  // first hidden row of the box
          if (lane == 0 && by < p.H) {  // H is a multiple of 64: a box lies wholly inside or past H
            const int bx = row_blk0 + c * 32;                               // token column
            if (t.chunk == 0)
              tma_store_2d(&map_dx, xstage, bx, by);
            else
              tma_reduce_add_2d(&map_dx, xstage, bx, by);
            bulk_commit_group();
          }
        } else if (t.kind == BK_DX) {
          // last chunk: this thread: hidden index h_dx; columns: token rows (compacted) row_blk0 + c * 32 + j
          if (h_dx < p.H) {
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] *= dscale;
            if (dx_prev) {
#pragma unroll
              for (int j = 0; j < 8; ++j) {
                v[4 * j] += pre[j].x;
                v[4 * j + 1] += pre[j].y;
                v[4 * j + 2] += pre[j].z;
                v[4 * j + 3] += pre[j].w;
              }
              if (c + 1 < c_hi) {  // the next 32 columns' sum, in flight during this chunk's work
#pragma unroll
                for (int j = 0; j < 8; ++j)
                  pre[j] = __ldcg(reinterpret_cast<const float4*>(acc_row + (c + 1) * 32) + j);
              }
            }
          }
          {
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
          // The warp's 32 rows x 32 columns leave by one TMA store of a 64-byte-swizzled box
          // (16-byte piece i of row r at position i ^ ((r / 2) % 4): conflict-free), through
          // two 2 KB halves of its slice used in turn; rows past the shard are clipped by TMA.
          const int h0 = t.n * BN + c * 32;
          const int v0 = t.m * P_RB + BM * static_cast<int>(rank) + q * 32;  // warp's first vocab row
          if (h0 < p.H && v0 < w) {
            uint8_t* half = xstage + ((c - c_lo) & 1) * 2048;
            if (c - c_lo >= 2 && lane == 0) bulk_wait_read_1();  // the box of two chunks ago has left it
            __syncwarp();
            uint4* row = reinterpret_cast<uint4*>(half + lane * 64);
#pragma unroll
            for (int i = 0; i < 4; ++i)
              row[i ^ ((lane >> 1) & 3)] =
                  make_uint4(pack2<BF16>(v[8 * i] * dscale, v[8 * i + 1] * dscale),
                             pack2<BF16>(v[8 * i + 2] * dscale, v[8 * i + 3] * dscale),
                             pack2<BF16>(v[8 * i + 4] * dscale, v[8 * i + 5] * dscale),
                             pack2<BF16>(v[8 * i + 6] * dscale, v[8 * i + 7] * dscale));
            fence_async_shared();
            __syncwarp();
            if (lane == 0) {
              tma_store_2d(&map_dw, half, h0, t.chunk * p.v_chunk + v0);
              bulk_commit_group();
            }
            dw_pending = true;
          }
        }
      }
      tc_fence_before();
      mbar_arrive_cluster(leader_tempty + 8u * acc);
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1u;
      }
      // publish: a GT tile per warp (each warp's G^T rows, counted 8 times per CTA), a DXT tile
      // per CTA (after all eight warps' TMA stores / adds); dW tiles have nothing to publish
      if (t.kind == BK_G) {
        __syncwarp();
        if (lane == 0) {
          __threadfence();
          atomicAdd(&gdone[t.chunk], 1);
        }
      } else if (t.kind == BK_DX) {
        if (!dx_last && lane == 0) {
          bulk_wait_all();       // this warp's TMA stores / adds of the tile are done in global memory
          fence_async_global();  // and ordered before the publishing thread's fence and count
        }
        named_bar<1, P_EPI>();  // all of this CTA's stores of the tile happen before its count
        if (et == 0) {
          const bool x_last = geo.xch && t.chunk + 1 == geo.C;
          if (x_last)
            __threadfence_system();
          else
            __threadfence();
          atomicAdd(&dxchain[t.m * geo.nh + t.n], 1);
          if (x_last)
            multimem_st_release_b32(p.x_flags_mc + p.x_world +
                                        ((static_cast<size_t>(t.m) * p.x_world + p.x_rank) * geo.nh + t.n) * 2 + rank,
                                    p.x_epoch);
        }
      }
      LMCE_PROF(const long long dwk = clock64() - pe_tile;
                if (t.kind == BK_G) { wk_g += dwk; ++n_g; } else if (t.kind == BK_DX) { wk_dx += dwk; ++n_dx; }
                else { wk_dw += dwk; ++n_dw; }
                if (tle) tle[7] = global_timer_ns();)
    }
    if (lane == 0) bulk_wait_all();  // no TMA store may still read the slice when the CTA exits
    if (!ok) {
      raise_error(p.err, ERR_TIMEOUT);
      *abort_flag = 1;
    }
    LMCE_PROF(if (et == 0) {
      prof_store(PS_E_SCHED, e_sched); prof_store(PS_E_CHAIN, e_chain); prof_store(PS_E_XCH, e_xch);
      prof_store(PS_E_TFULL_G, tf_g); prof_store(PS_E_TFULL_DX, tf_dx); prof_store(PS_E_TFULL_DW, tf_dw);
      prof_store(PS_E_WORK_G, wk_g); prof_store(PS_E_WORK_DX, wk_dx); prof_store(PS_E_WORK_DW, wk_dw);
      prof_store(PS_E_N_G, n_g); prof_store(PS_E_N_DX, n_dx); prof_store(PS_E_N_DW, n_dw);
      prof_store(PS_E_LOOP, clock64() - pl0);
    })
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
  LMCE_PROF(if (threadIdx.x == 0) prof_store(PS_TOTAL, clock64() - prof_t_begin);)
  if (warp == 1) {
    __syncwarp();
    tmem_dealloc_pair(tmem_base, TMEM_COLS);
  }
}

}  // namespace lmce
