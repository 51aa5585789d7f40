// Persistent backward of the lm_head CE head: one launch computes dX and dW.
//
// The vocabulary is cut into chunks of v_chunk rows. For chunk c three kinds of
// 128x256 output tiles exist:
//   G(c)   recomputed logits tile X_lab . W_c^T -> G = (softmax - onehot) * 2^15
//          in the input dtype, written to G buffer c % NUM_GBUF
//          (replaces the reference's pass-2 GEMM + lm_head_piece_kernel MODE 1,
//          solution/ops.py:287-319, solution/kernels.py:517-531)
//   DX(c)  dX_tile += G_c . W_c (K = chunk width); fp32 accumulation across chunks
//          in chunk order; the last chunk scales by grad_loss / denom / 2^15 and
//          scatters rows to token order (replaces ops.py:320 and 337-338)
//   DW(c)  dW rows of chunk c = G_c^T . X_lab (K = labelled tokens); new, the
//          reference returns None for the weight (ops.py:339)
// All tiles of the whole backward form one list, claimed in order through an
// atomic ticket by persistent CTAs (one per SM):
//   G(0) G(1) DX(0) DW(0) G(2) DX(1) DW(1) ... G(C-1) DX(C-2) DW(C-2) DX(C-1) DW(C-1)
// with device-side dependencies checked by the TMA producer before it loads a tile:
//   DX(c), DW(c) wait for all G(c) tiles (gdone[c]);
//   G(c) waits until the DX/DW tiles of chunk c - NUM_GBUF released its buffer (consumed[]);
//   DX(c) tile (m,n) waits for DX(c-1) tile (m,n) (dxchain[]), keeping the fp32
//   read-modify-write of dX in chunk order (deterministic, no atomics on data).
// A tile only waits for tiles earlier in the list, and tiles are claimed in list
// order by running CTAs, so the earliest unfinished tile can always progress.
//
// Vocab-sharded runs over NVLink SHARP add a fourth kind, the cross-GPU dX sum:
//   XCH(m, q)  rows of block m, columns piece q of this rank's slice of H: once every
//              rank has written its last-chunk dX rows of block m, read the sum over
//              the GPUs with multimem.ld_reduce and store it, in the input dtype, to
//              every GPU's output copy with multimem.st.
// The tail of the list then becomes DX(C-1) XCH DW(C-2) DW(C-1), so the exchange runs
// while the last two chunks' dW tiles still compute. XCH waits only for DX tiles,
// which every rank lists before its own XCH items, so no cycle between ranks exists.
// Signals are words of a multicast flag array stamped with the call's epoch (so they
// need no reset, whatever rows a call has): slot (m, rank, n) when DX(C-1) tile (m, n)
// of that rank is written, and slot `rank` once all of the rank's XCH items are done.
// Before the kernel ends, CTA 0 waits for every rank's done slot: then no GPU still
// reads this rank's partials, and every GPU's sums have landed in this rank's copy.
// Producers of a dependency publish with stores -> CTA barrier -> fence ->
// atomic add; consumers acquire the counter, then fence the async proxy before
// their TMA reads of G. Every wait is bounded.
#pragma once

#include "lmce_engine.cuh"

namespace lmce {

constexpr int NUM_GBUF = 3;
// G is stored prescaled by 2^15 in the input dtype: p * dnll for p ~ 1/V would underflow
// fp16 otherwise, and |G| <= 2^15 keeps it finite (the reference's 2^16 could overflow at
// denom 1). The dX / dW epilogues divide it out.
constexpr float GSCALE = 32768.0f;
constexpr float GSCALE_LOG2 = 15.0f;
constexpr int SCHED_DEPTH = 4;
// Per-warp staging of 32 rows x 32 columns of 16-bit output (64 bytes a row, padded to
// 80 so the row-wise 16-byte writes of a warp hit distinct banks).
constexpr int ROW_STAGE_PITCH = 80;
constexpr int ROW_STAGE_BYTES = 4 * 32 * ROW_STAGE_PITCH;  // 10 KB for the four epilogue warps
constexpr int BWD_SMEM_BYTES = TileCfg<false>::SMEM_BYTES + ROW_STAGE_BYTES;
constexpr int XCH_COLS = 256;   // columns of one exchange item
constexpr int XCH_UNROLL = 4;   // independent 32-byte reductions in flight per thread

enum : int { BK_END = -1, BK_G = 0, BK_DX = 1, BK_DW = 2, BK_XCH = 3 };

struct BwdTile {
  int kind, chunk, m, n;
};

struct BwdParams {
  int rows_pad;            // allocated rows of X_lab and of each G buffer (multiple of 128)
  int H;                   // hidden size
  int V;                   // vocab rows of this shard
  int v_chunk;             // chunk width (multiple of 256)
  int n_chunks;
  const int* count;        // device: number of labelled tokens (compacted rows)
  const int* lbl_lab;      // per compacted row: label local to the shard, -1 if elsewhere
  const float* lse_lab;    // per compacted row: lse
  void* g;                 // G buffers [NUM_GBUF][rows_pad][v_chunk], input dtype
  float* dx_acc;           // fp32 [rows_pad][H], compacted row order
  const int* row_idx;      // compacted row -> token row
  void* dx_out;            // [N][H] input dtype (nullable)
  float* dx_out_f32;       // [N][H] fp32 (nullable; vocab-sharded runs: this rank's contribution)
  // fused cross-GPU dX sum (x_flags_mc == nullptr: off); dx_out_f32 is then the local
  // view of the symmetric partial buffer whose multicast address is x_part_mc
  const float* x_part_mc;  // multicast [N][H] fp32 partials
  void* x_out_mc;          // multicast [N][H] input dtype: the sums
  const uint32_t* x_flags; // local view of the flags: [world] done slots, then [m][world][num_hn] tile slots
  uint32_t* x_flags_mc;    // multicast view of the flags
  uint32_t x_epoch;        // stamp of this call (same on every rank)
  int x_rank, x_world;
  int x_lo, x_hi;          // this rank's column slice of H (multiples of 8)
  void* dw_out;            // [V][H] input dtype (nullable)
  int want_dx, want_dw;
  int mn3_h;               // X and W MN-major maps are 3-D (H a multiple of 64, H >= 256); G's always are
  const float* grad_loss;  // device scalar (nullable: 1)
  const float* denom;      // device scalar
  float gscale;            // G prescale
  int* sync;               // zeroed: [0] ticket, [1..C] gdone, [1+C..2C] consumed, [1+2C..] dxchain,
                           // then one count of this rank's finished XCH items
  int* err;
  unsigned long long timeout_ns;
};

// Geometry derived from the parameters and the device-side labelled-token count
// (identical in every thread of every CTA).
struct BwdGeom {
  int n_lab, num_m, num_hn, C, vc, V, nX;
  bool dx, dw, xch;  // xch: the cross-GPU exchange is on (this rank may still own no XCH items)
  __device__ __forceinline__ int width(int c) const { return min(vc, V - c * vc); }
  __device__ __forceinline__ int nG(int c) const { return num_m * ((width(c) + BN - 1) / BN); }
  __device__ __forceinline__ int nDX() const { return dx ? num_m * num_hn : 0; }
  __device__ __forceinline__ int nDW(int c) const { return dw ? ((width(c) + BM - 1) / BM) * num_hn : 0; }
  __device__ __forceinline__ int num_kb(const BwdTile& t, int H) const {
    if (t.kind == BK_XCH) return 0;
    if (t.kind == BK_G) return (H + BK - 1) / BK;
    if (t.kind == BK_DX) return (width(t.chunk) + BK - 1) / BK;
    return (n_lab + BK - 1) / BK;
  }
};

__device__ __forceinline__ BwdGeom make_geom(const BwdParams& p) {
  BwdGeom g;
  g.n_lab = *p.count;
  g.num_m = (g.n_lab + BM - 1) / BM;
  g.num_hn = (p.H + BN - 1) / BN;
  g.C = p.n_chunks;
  g.vc = p.v_chunk;
  g.V = p.V;
  g.dx = p.want_dx != 0;
  g.dw = p.want_dw != 0;
  g.xch = p.x_flags_mc != nullptr && g.dx;
  g.nX = g.xch ? g.num_m * ((p.x_hi - p.x_lo + XCH_COLS - 1) / XCH_COLS) : 0;
  return g;
}

// Decoder of the tile list (see the file comment). Segments are walked with a
// forward-only cursor: one producer thread asks for increasing ticket numbers,
// so the total walking over a launch is one pass over the ~3C segments.
struct TileCursor {
  int seg;             // segment index: 0 = G(0); then 3 per chunk c: G(c+1), DX(c), DW(c)
  long long seg_start; // first ticket of segment `seg`

  __device__ __forceinline__ void init() {
    seg = 0;
    seg_start = 0;
  }

  // kind, chunk, count and m-extent of segment `s`; false past the last segment
  __device__ __forceinline__ static bool segment(const BwdGeom& g, int s, int& kind, int& chunk, int& count,
                                                 int& mdim) {
    if (g.xch) {
      // exchange order: after DX(C-2) (after G(0) when C == 1): DX(C-1) XCH DW(C-2) DW(C-1)
      const int head = g.C >= 2 ? 3 * g.C - 3 : 1;
      if (s >= head) {
        const int u = s - head;
        chunk = g.C - 1;
        mdim = g.num_m;
        if (u == 0) {
          kind = BK_DX;
          count = g.nDX();
        } else if (u == 1) {
          kind = BK_XCH;
          count = g.nX;
        } else if (u <= 3) {
          kind = BK_DW;
          chunk = g.C - 4 + u;  // C-2, then C-1
          count = chunk >= 0 ? g.nDW(chunk) : 0;
          mdim = chunk >= 0 ? (g.width(chunk) + BM - 1) / BM : 1;
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
      mdim = g.num_m;
      return true;
    }
    const int c = (s - 1) / 3, r = (s - 1) % 3;
    if (c >= g.C) return false;
    if (r == 0) {
      kind = BK_G;
      chunk = c + 1;
      count = c + 1 < g.C ? g.nG(c + 1) : 0;
      mdim = g.num_m;
    } else if (r == 1) {
      kind = BK_DX;
      chunk = c;
      count = g.nDX();
      mdim = g.num_m;
    } else {
      kind = BK_DW;
      chunk = c;
      count = g.nDW(c);
      mdim = (g.width(c) + BM - 1) / BM;
    }
    return true;
  }

  // Tile of ticket t (t never decreases between calls); false past the end of the list.
  __device__ __forceinline__ bool decode(const BwdGeom& g, long long t, BwdTile& out) {
    for (;;) {
      int kind, chunk, count, mdim;
      if (!segment(g, seg, kind, chunk, count, mdim)) return false;
      if (t < seg_start + count) {
        const int i = static_cast<int>(t - seg_start);
        out.kind = kind;
        out.chunk = chunk;
        out.m = i % mdim;
        out.n = i / mdim;
        return true;
      }
      seg_start += count;
      ++seg;
    }
  }
};

// Read a schedule-ring entry written by the producer thread (after the sched_full wait).
__device__ __forceinline__ BwdTile read_ring(const BwdTile* e) {
  const volatile int* v = reinterpret_cast<const volatile int*>(e);
  BwdTile t;
  t.kind = v[0];
  t.chunk = v[1];
  t.m = v[2];
  t.n = v[3];
  return t;
}

__device__ __forceinline__ int ld_acquire_gpu(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Bounded wait until *p >= target (acquire). False on timeout or abort.
__device__ __forceinline__ bool wait_counter(const int* p, int target, volatile int* abort, uint64_t limit_ns) {
  if (ld_acquire_gpu(p) >= target) return true;
  const uint64_t t0 = global_timer_ns();
  for (;;) {
    __nanosleep(128);
    if (ld_acquire_gpu(p) >= target) return true;
    if (*abort) return false;
    if (global_timer_ns() - t0 > limit_ns) return false;
  }
}

// Publish: all 128 epilogue threads' global stores happen before the increment.
__device__ __forceinline__ void publish_add(int* ctr, int v) {
  epilogue_bar();
  if (threadIdx.x == EPI_THREAD0) {
    __threadfence();
    atomicAdd(ctr, v);
  }
}

// Store a 32-row x 32-column block of 16-bit values held one row per lane (v = this
// lane's 32 values) to rows [row0, row0 + 32) of a row-major tensor with `pitch`
// elements per row, through the warp's staging slice: each store instruction then
// covers 8 rows x 64 contiguous bytes instead of 32 rows x 16 bytes. Rows for which
// `row_ok(r)` is false are not written. Called by all 32 lanes of the warp.
template <bool BF16, typename RowOk>
__device__ __forceinline__ void store_rows32(uint8_t* stage, const float* v, char* base, size_t pitch_bytes,
                                             int row0, int lane, RowOk row_ok) {
  uint4* mine = reinterpret_cast<uint4*>(stage + lane * ROW_STAGE_PITCH);
#pragma unroll
  for (int q = 0; q < 4; ++q)
    mine[q] = make_uint4(pack2<BF16>(v[8 * q + 0], v[8 * q + 1]), pack2<BF16>(v[8 * q + 2], v[8 * q + 3]),
                         pack2<BF16>(v[8 * q + 4], v[8 * q + 5]), pack2<BF16>(v[8 * q + 6], v[8 * q + 7]));
  __syncwarp();
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int r = i * 8 + (lane >> 2);
    const int piece = lane & 3;
    const uint4 u = *reinterpret_cast<const uint4*>(stage + r * ROW_STAGE_PITCH + piece * 16);
    if (row_ok(row0 + r)) *reinterpret_cast<uint4*>(base + static_cast<size_t>(row0 + r) * pitch_bytes + piece * 16) = u;
  }
  __syncwarp();
}

// Bounded wait until the word at f reaches stamp `target` (wrapping compare, system-scope acquire).
__device__ __forceinline__ bool wait_flag_sys(const uint32_t* f, uint32_t target, volatile int* abort,
                                              uint64_t limit_ns) {
  if (static_cast<int>(ld_acquire_sys_u32(f) - target) >= 0) return true;
  const uint64_t t0 = global_timer_ns();
  for (;;) {
    __nanosleep(256);
    if (static_cast<int>(ld_acquire_sys_u32(f) - target) >= 0) return true;
    if (*abort) return false;
    if (global_timer_ns() - t0 > limit_ns) return false;
  }
}

// Exchange item XCH(m, q), run by the 128 epilogue threads: the cross-GPU sum of
// dX rows [row0, row0 + 128) of row block m (clipped to n_lab) over columns
// [c_lo, c_hi), written in the input dtype to every GPU's output copy. It starts once
// every rank stamped the `stamps` flag slots it owns for block m (one per DX tile
// half that covers the block). Consecutive threads take consecutive 8-column groups
// of a row, so each warp instruction covers contiguous bytes. The call that brings
// this GPU's count of finished items to `items` stamps the GPU's done slot. Run by the
// 128 threads EPI_THREAD0 .. EPI_THREAD0 + 127, which synchronise on named barrier BAR.
template <bool BF16, int BAR>
__device__ __forceinline__ void exchange_rows_range(const BwdParams& p, int row0, int n_lab, int stamps,
                                                    const BwdTile& t, int* xdone, int items, volatile int* abort_flag,
                                                    uint64_t tlimit) {
  const int et = static_cast<int>(threadIdx.x) - EPI_THREAD0;
  const int slots = p.x_world * stamps;
  const uint32_t* block_slots = p.x_flags + p.x_world + static_cast<size_t>(t.m) * slots;
  for (int i = et; i < slots; i += EPI_THREADS) {
    if (!wait_flag_sys(block_slots + i, p.x_epoch, abort_flag, tlimit)) {
      raise_error(p.err, ERR_TIMEOUT);
      *abort_flag = 1;
      break;
    }
  }
  if (!named_bar_all<BAR, EPI_THREADS>(*abort_flag == 0)) return;  // same decision in all 128 threads
  const int c_lo = p.x_lo + t.n * XCH_COLS;
  const int c_hi = min(c_lo + XCH_COLS, p.x_hi);
  const int groups = (c_hi - c_lo) / 8;
  const int rows = max(0, min(BM, n_lab - row0));
  const int total = rows * groups;
  for (int base = 0; base < total; base += EPI_THREADS * XCH_UNROLL) {
    float4 lo[XCH_UNROLL], hi[XCH_UNROLL];
    long long off[XCH_UNROLL];
#pragma unroll
    for (int u = 0; u < XCH_UNROLL; ++u) {
      const int i = base + u * EPI_THREADS + et;
      off[u] = -1;
      if (i < total) {
        const int r = i / groups;
        const int g = i - r * groups;
        off[u] = static_cast<long long>(p.row_idx[row0 + r]) * p.H + c_lo + g * 8;
        lo[u] = multimem_ld_reduce_add_v4_f32(p.x_part_mc + off[u]);
        hi[u] = multimem_ld_reduce_add_v4_f32(p.x_part_mc + off[u] + 4);
      }
    }
#pragma unroll
    for (int u = 0; u < XCH_UNROLL; ++u) {
      if (off[u] >= 0)
        multimem_st_v4_x2<BF16>(static_cast<char*>(p.x_out_mc) + off[u] * 2, pack2<BF16>(lo[u].x, lo[u].y),
                                pack2<BF16>(lo[u].z, lo[u].w), pack2<BF16>(hi[u].x, hi[u].y),
                                pack2<BF16>(hi[u].z, hi[u].w));
    }
  }
  __threadfence_system();
  named_bar<BAR, EPI_THREADS>();
  if (et == 0) {
    const int prev = atomicAdd(xdone, 1);
    if (prev + 1 == items) {
      __threadfence_system();
      multimem_st_release_b32(p.x_flags_mc + p.x_rank, p.x_epoch);
    }
  }
}

// UMMA k-loop of one tile. The operand majors and the instruction descriptor are
// template constants: tcgen05.mma takes them from uniform registers, and values
// that depend on the tile kind read from shared memory are not provably uniform
// (the compiler then serialises every issue, halving the tensor-pipe rate).
template <bool BF16, bool A_MN, bool B_MN, int STAGES>
__device__ __forceinline__ bool mma_tile(uint8_t* smem, uint64_t* full_bar, uint64_t* empty_bar, int nkb,
                                         uint32_t d_tmem, int& stage, uint32_t& phase, volatile int* abort_flag,
                                         uint64_t tlimit) {
  using C = TileCfg<false>;
  constexpr uint32_t idesc = make_idesc_f16(BF16, A_MN, B_MN, BM, BN);
  for (int kb = 0; kb < nkb; ++kb) {
    if (!mbar_wait(&full_bar[stage], phase, abort_flag, tlimit)) return false;
    tc_fence_after();
    const uint32_t sa = smem_u32(smem + stage * C::STAGE_BYTES);
#pragma unroll
    for (int k = 0; k < BK / UMMA_K; ++k)
      umma_f16_ss(d_tmem, operand_desc(sa, A_MN, k), operand_desc(sa + C::A_BYTES, B_MN, k), idesc,
                  (kb | k) != 0 ? 1u : 0u);
    umma_commit(&empty_bar[stage]);
    if (++stage == STAGES) {
      stage = 0;
      phase ^= 1u;
    }
  }
  return true;
}

template <bool BF16, int STAGES>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    lmce_bwd_kernel(const __grid_constant__ CUtensorMap map_xk, const __grid_constant__ CUtensorMap map_xmn,
                    const __grid_constant__ CUtensorMap map_wk, const __grid_constant__ CUtensorMap map_wmn,
                    const __grid_constant__ CUtensorMap map_gk, const __grid_constant__ CUtensorMap map_gmn,
                    const BwdParams p) {
  using C = TileCfg<false>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + STAGES * C::STAGE_BYTES);
  uint64_t* empty_bar = full_bar + STAGES;
  uint64_t* tfull_bar = empty_bar + STAGES;
  uint64_t* tempty_bar = tfull_bar + 2;
  uint64_t* drain_bar = tempty_bar + 2;
  uint64_t* sched_full = drain_bar + 1;
  uint64_t* sched_empty = sched_full + SCHED_DEPTH;
  BwdTile* ring = reinterpret_cast<BwdTile*>(sched_empty + SCHED_DEPTH);
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(ring + SCHED_DEPTH);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = __shfl_sync(0xffffffffu, threadIdx.x / 32, 0);
  const int lane = threadIdx.x & 31;
  // epilogue row staging (after the barrier block); warp quadrant q uses slice q
  uint8_t* row_stage = smem + STAGES * C::STAGE_BYTES + 1024 + (warp & 3) * 32 * ROW_STAGE_PITCH;
  const BwdGeom geo = make_geom(p);
  int* ticket = p.sync;
  int* gdone = p.sync + 1;
  int* consumed = p.sync + 1 + p.n_chunks;
  int* dxchain = p.sync + 1 + 2 * p.n_chunks;
  int* xdone = dxchain + (p.rows_pad / BM) * geo.num_hn;

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
    for (int s = 0; s < SCHED_DEPTH; ++s) {
      mbar_init(&sched_full[s], 1);
      mbar_init(&sched_empty[s], 1 + EPI_THREADS);  // UMMA lane + epilogue threads
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&map_xk);
    tma_prefetch_desc(&map_xmn);
    tma_prefetch_desc(&map_wk);
    tma_prefetch_desc(&map_wmn);
    tma_prefetch_desc(&map_gk);
    tma_prefetch_desc(&map_gmn);
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
    // ------------------------------------------- scheduler + TMA producer ---
    if (lane == 0) {
      int stage = 0, slot = 0;
      uint32_t phase = 0, sphase = 0;
      int issued = 0;
      bool ok = true;
      TileCursor cur;
      cur.init();
      int g_ready_chunk = -1;    // highest chunk whose G tiles this producer saw complete
      int gbuf_free_chunk = -1;  // highest chunk whose G buffer this producer saw released
      int next_ticket = atomicAdd(ticket, 1);  // claimed one tile ahead of its loads
      for (;;) {
        if (!mbar_wait(&sched_empty[slot], sphase ^ 1u, abort_flag, tlimit)) {
          ok = false;
          break;
        }
        BwdTile t;
        const bool has = cur.decode(geo, next_ticket, t);
        if (!has) t.kind = BK_END;
        {
          volatile int* e = reinterpret_cast<volatile int*>(&ring[slot]);
          e[0] = t.kind;
          e[1] = t.chunk;
          e[2] = t.m;
          e[3] = t.n;
        }
        mbar_arrive(&sched_full[slot]);
        if (++slot == SCHED_DEPTH) {
          slot = 0;
          sphase ^= 1u;
        }
        if (!has) break;
        next_ticket = atomicAdd(ticket, 1);  // result is first needed after this tile's loads

        // Dependencies of this tile. Tiles of one chunk are contiguous in the list, so a
        // dependency seen satisfied once is remembered and later tiles skip the acquire.
        const int gbuf = t.chunk % NUM_GBUF;
        if (t.kind == BK_G) {
          if (t.chunk >= NUM_GBUF && t.chunk > gbuf_free_chunk) {
            const int prev = t.chunk - NUM_GBUF;
            ok = wait_counter(&consumed[prev], geo.nDX() + geo.nDW(prev), abort_flag, tlimit);
            if (ok) gbuf_free_chunk = t.chunk;
          }
        } else if (t.kind != BK_XCH) {
          bool acquired = false;
          if (t.chunk > g_ready_chunk) {
            ok = wait_counter(&gdone[t.chunk], geo.nG(t.chunk), abort_flag, tlimit);
            if (ok) g_ready_chunk = t.chunk;
            acquired = true;
          }
          if (ok && t.kind == BK_DX && t.chunk > 0) {
            ok = wait_counter(&dxchain[t.m * geo.num_hn + t.n], t.chunk, abort_flag, tlimit);
            acquired = true;
          }
          // G and dX were written by generic stores of other CTAs; order them before the async-proxy reads
          if (acquired) asm volatile("fence.proxy.async.global;" ::: "memory");
        }
        if (!ok) break;

        const int nkb = geo.num_kb(t, p.H);
        for (int kb = 0; kb < nkb; ++kb) {
          if (!mbar_wait(&empty_bar[stage], phase ^ 1u, abort_flag, tlimit)) {
            ok = false;
            break;
          }
          uint8_t* sa = smem + stage * C::STAGE_BYTES;
          uint8_t* sb = sa + C::A_BYTES;
          uint64_t* fb = &full_bar[stage];
          mbar_arrive_expect_tx(fb, C::STAGE_BYTES);
          const int k0 = kb * BK;
          if (t.kind == BK_G) {
            load_operand<BM>(sa, &map_xk, fb, false, t.m * BM, k0);
            load_operand<BN>(sb, &map_wk, fb, false, t.chunk * p.v_chunk + t.n * BN, k0);
          } else if (t.kind == BK_DX) {
            load_operand<BM>(sa, &map_gk, fb, false, gbuf * p.rows_pad + t.m * BM, k0);
            if (p.mn3_h)
              load_operand_mn3<BN>(sb, &map_wmn, fb, t.n * BN, t.chunk * p.v_chunk + k0);
            else
              load_operand<BN>(sb, &map_wmn, fb, true, t.n * BN, t.chunk * p.v_chunk + k0);
          } else {
            load_operand_mn3<BM>(sa, &map_gmn, fb, t.m * BM, gbuf * p.rows_pad + k0);
            if (p.mn3_h)
              load_operand_mn3<BN>(sb, &map_xmn, fb, t.n * BN, k0);
            else
              load_operand<BN>(sb, &map_xmn, fb, true, t.n * BN, k0);
          }
          ++issued;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
      }
      if (!ok) {
        raise_error(p.err, ERR_TIMEOUT);
        *abort_flag = 1;
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
        if (!mbar_wait(&tempty_bar[acc], acc_phase ^ 1u, abort_flag, tlimit)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
        const int nkb = geo.num_kb(t, p.H);
        if (t.kind == BK_G)
          ok = mma_tile<BF16, false, false, STAGES>(smem, full_bar, empty_bar, nkb, d_tmem, stage, phase, abort_flag,
                                                     tlimit);
        else if (t.kind == BK_DX)
          ok = mma_tile<BF16, false, true, STAGES>(smem, full_bar, empty_bar, nkb, d_tmem, stage, phase, abort_flag,
                                                    tlimit);
        else
          ok = mma_tile<BF16, true, true, STAGES>(smem, full_bar, empty_bar, nkb, d_tmem, stage, phase, abort_flag,
                                                   tlimit);
        if (!ok) break;
        umma_commit(&tfull_bar[acc]);  // also fires when nkb == 0 (no UMMA issued)
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
      if (!ok) {
        raise_error(p.err, ERR_TIMEOUT);
        *abort_flag = 1;
      }
      umma_commit(drain_bar);
      volatile int no_abort = 0;
      mbar_wait(drain_bar, 0, &no_abort, tlimit);
    }
  } else {
    // ---------------------------------------------------------- epilogue ---
    const int q = warp & 3;
    const int r_in_tile = q * 32 + lane;
    const uint32_t lane_base = static_cast<uint32_t>(q * 32) << 16;
    const float gl = p.grad_loss ? *p.grad_loss : 1.0f;
    const float dscale = gl / (*p.denom) / p.gscale;
    int slot = 0, acc = 0;
    uint32_t sphase = 0, acc_phase = 0;
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
      if (t.kind == BK_XCH) {
        if (!mbar_wait(&tfull_bar[acc], acc_phase, abort_flag, tlimit)) {  // no UMMA: only keeps the slot order
          ok = false;
          break;
        }
        exchange_rows_range<BF16, 1>(p, t.m * BM, geo.n_lab, geo.num_hn, t, xdone, geo.nX, abort_flag, tlimit);
        mbar_arrive(&tempty_bar[acc]);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1u;
        }
        continue;
      }
      const bool have_acc = geo.num_kb(t, p.H) > 0;
      const int w = geo.width(t.chunk);
      const int row = t.m * BM + r_in_tile;

      // per-row inputs of a G tile
      int lbl = -1;
      float lseL = 0.f;
      const bool g_row_ok = row < geo.n_lab;
      if (t.kind == BK_G && g_row_ok) {
        const int y = p.lbl_lab[row];
        lbl = y >= 0 ? y - t.chunk * p.v_chunk : -1;
        lseL = p.lse_lab[row] * LOG2E;
      }
      if (t.kind == BK_DX && t.chunk > 0) {
        // dX rows of this tile were last written by DX(chunk-1) on some CTA.
        if (threadIdx.x == EPI_THREAD0 &&
            !wait_counter(&dxchain[t.m * geo.num_hn + t.n], t.chunk, abort_flag, tlimit)) {
          raise_error(p.err, ERR_TIMEOUT);
          *abort_flag = 1;
        }
        epilogue_bar();
      }
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
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = have_acc ? __uint_as_float(raw[j]) : 0.0f;
        const int col0 = t.n * BN + c * 32;

        if (t.kind == BK_G) {
          // G = (softmax - onehot) * 2^15 on the dtype-rounded logits; 0 outside the chunk / labelled rows
          const unsigned rel = static_cast<unsigned>(lbl - col0);
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const float z = round_to_input<BF16>(v[j]);
            float pr = ex2_approx(fmaf(z, LOG2E, -lseL));
            if (static_cast<unsigned>(j) == rel) pr -= 1.0f;
            v[j] = (g_row_ok && col0 + j < w) ? pr * p.gscale : 0.0f;
          }
          char* gbase = reinterpret_cast<char*>(p.g) +
                        (static_cast<size_t>(t.chunk % NUM_GBUF) * p.rows_pad * p.v_chunk + col0) * 2;
          store_rows32<BF16>(row_stage, v, gbase, static_cast<size_t>(p.v_chunk) * 2, t.m * BM + q * 32, lane,
                             [](int) { return true; });
        } else if (t.kind == BK_DX) {
          if (row < geo.n_lab && col0 < p.H) {
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] *= dscale;
            float* accp = p.dx_acc + static_cast<size_t>(row) * p.H + col0;
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
            } else {
              const size_t trow = static_cast<size_t>(p.row_idx[row]);
              if (p.dx_out_f32 != nullptr) {
                float* dst = p.dx_out_f32 + trow * p.H + col0;
#pragma unroll
                for (int j = 0; j < 32; j += 4)
                  *reinterpret_cast<float4*>(dst + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
              }
              if (p.dx_out != nullptr) store32_dtype<BF16>(reinterpret_cast<char*>(p.dx_out) + (trow * p.H + col0) * 2, v);
            }
          }
        } else {  // BK_DW
          if (col0 < p.H) {
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] *= dscale;
            char* dbase = reinterpret_cast<char*>(p.dw_out) +
                          (static_cast<size_t>(t.chunk) * p.v_chunk * p.H + col0) * 2;
            store_rows32<BF16>(row_stage, v, dbase, static_cast<size_t>(p.H) * 2, t.m * BM + q * 32, lane,
                               [w](int r) { return r < w; });
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&tempty_bar[acc]);
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1u;
      }
      // publish completion for dependent tiles
      if (t.kind == BK_G) {
        publish_add(&gdone[t.chunk], 1);
      } else if (t.kind == BK_DX) {
        epilogue_bar();
        if (threadIdx.x == EPI_THREAD0) {
          const bool x_last = geo.xch && t.chunk + 1 == geo.C;
          if (x_last)
            __threadfence_system();  // the partial rows are read by every GPU's exchange items
          else
            __threadfence();
          atomicAdd(&dxchain[t.m * geo.num_hn + t.n], 1);
          atomicAdd(&consumed[t.chunk], 1);
          if (x_last)
            multimem_st_release_b32(
                p.x_flags_mc + p.x_world + (static_cast<size_t>(t.m) * p.x_world + p.x_rank) * geo.num_hn + t.n,
                p.x_epoch);
        }
      } else {
        publish_add(&consumed[t.chunk], 1);
      }
    }
    if (!ok) {
      raise_error(p.err, ERR_TIMEOUT);
      *abort_flag = 1;
    }
    if (geo.xch && blockIdx.x == 0) {
      // a rank without XCH items is done at once; then wait for every rank's done stamp
      const int et = static_cast<int>(threadIdx.x) - EPI_THREAD0;
      if (et == 0 && geo.nX == 0) multimem_st_release_b32(p.x_flags_mc + p.x_rank, p.x_epoch);
      for (int r = et; r < p.x_world; r += EPI_THREADS) {
        if (!*abort_flag && !wait_flag_sys(p.x_flags + r, p.x_epoch, abort_flag, tlimit)) {
          raise_error(p.err, ERR_TIMEOUT);
          *abort_flag = 1;
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) {
    __syncwarp();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

}  // namespace lmce
