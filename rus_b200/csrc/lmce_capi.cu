// C-ABI, launch code and the small auxiliary kernels of the lm_head CE head.
//
// Host responsibilities here: argument validation, TMA tensor-map encoding,
// schedule sizing (vocab slabs, vocab chunks), and stream-ordered launches.
// Nothing in this file allocates device memory or synchronises the stream.
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <atomic>
#include <mutex>
#include <utility>

#include "../../include/lmce.h"
#include "lmce_bwd.cuh"
#include "lmce_bwd_pair.cuh"
#include "lmce_pack.cuh"
#include "lmce_embed.cuh"
#include "lmce_rmsnorm.cuh"

using namespace lmce;

static_assert(sizeof(Part) == sizeof(lmce_part), "record layout mismatch");

// Library-wide device error word (one instance per device).
__device__ int g_lmce_err;

namespace {

thread_local char t_err[512] = "";
std::atomic<unsigned long long> g_launches{0};
// Process-wide (not per thread): autograd runs backward passes on its own worker thread.
std::atomic<CUevent> g_timing[2][2] = {{{nullptr}, {nullptr}}, {{nullptr}, {nullptr}}};
PFN_cuEventRecord_v2000 g_event_record = nullptr;

// Records the benchmark timing event of slot `which` (edge 0 begin / 1 end), if set.
// The driver call is used because the events usually come from another runtime
// instance in the process (the caller's framework); driver handles are shared.
void timing_mark(int which, int edge, cudaStream_t st) {
  CUevent ev = g_timing[which][edge].load(std::memory_order_acquire);
  if (ev != nullptr && g_event_record != nullptr) g_event_record(ev, reinterpret_cast<CUstream>(st));
}

// Every kernel launch in this file goes through this check, which also counts it.
int launched() {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    std::snprintf(t_err, sizeof(t_err), "kernel launch failed: %s", cudaGetErrorString(e));
    return LMCE_ERR_CUDA;
  }
  g_launches.fetch_add(1, std::memory_order_relaxed);
  return LMCE_OK;
}

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(t_err, sizeof(t_err), fmt, ap);
  va_end(ap);
  return code;
}

#define LMCE_CUDA(expr)                                                                         \
  do {                                                                                          \
    cudaError_t e_ = (expr);                                                                    \
    if (e_ != cudaSuccess) return fail(LMCE_ERR_CUDA, "%s: %s", #expr, cudaGetErrorString(e_)); \
  } while (0)

// ------------------------------------------------------------ device info ---

struct DevInfo {
  int sms = 0;
  int major = 0, minor = 0;
  int* err_ptr = nullptr;
  bool ok = false;
};

constexpr int kMaxDevices = 64;
DevInfo g_dev[kMaxDevices];
std::mutex g_dev_mu;

int device_info(DevInfo** out) {
  int dev = 0;
  LMCE_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) return fail(LMCE_ERR_UNSUPPORTED, "device ordinal %d out of range", dev);
  std::lock_guard<std::mutex> lk(g_dev_mu);
  DevInfo& d = g_dev[dev];
  if (!d.ok) {
    LMCE_CUDA(cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev));
    LMCE_CUDA(cudaDeviceGetAttribute(&d.major, cudaDevAttrComputeCapabilityMajor, dev));
    LMCE_CUDA(cudaDeviceGetAttribute(&d.minor, cudaDevAttrComputeCapabilityMinor, dev));
    if (d.major != 10 || d.minor != 0)
      return fail(LMCE_ERR_UNSUPPORTED, "lmce is built for sm_100a (B200); device %d is sm_%d%d", dev, d.major,
                  d.minor);
    void* p = nullptr;
    LMCE_CUDA(cudaGetSymbolAddress(&p, g_lmce_err));
    d.err_ptr = static_cast<int*>(p);
    d.ok = true;
  }
  *out = &d;
  return LMCE_OK;
}

unsigned long long wait_timeout_ns() {
  static unsigned long long v = [] {
    const char* s = std::getenv("LMCE_WAIT_TIMEOUT_MS");
    unsigned long long ms = s ? std::strtoull(s, nullptr, 10) : 4000ull;
    if (ms == 0) ms = 4000ull;
    return ms * 1000000ull;
  }();
  return v;
}

// ------------------------------------------------------------ tensor maps ---

PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

int get_encoder() {
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void* fn = nullptr;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
    if (e == cudaSuccess && q == cudaDriverEntryPointSuccess && fn != nullptr)
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  });
  return g_encode ? LMCE_OK : fail(LMCE_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
}

// Row-major 2-D tensor [outer][inner] of 16-bit elements, 128-byte swizzle, box {64, box_outer}.
int make_map(CUtensorMap* m, const void* base, bool bf16, uint64_t inner, uint64_t outer, uint64_t ld_elems,
             uint32_t box_outer) {
  if (reinterpret_cast<uintptr_t>(base) % 16 != 0) return fail(LMCE_ERR_INVALID_ARGUMENT, "tensor base not 16B aligned");
  if ((ld_elems * 2) % 16 != 0) return fail(LMCE_ERR_INVALID_ARGUMENT, "row stride not a multiple of 16 bytes");
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {ld_elems * 2};
  cuuint32_t box[2] = {64, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode(m, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                        const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(LMCE_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", static_cast<int>(r));
  return LMCE_OK;
}

// The same [outer][inner] tensor seen as 3-D for MN-major operands: {64 elements,
// outer (the k rows), inner / 64 blocks of 64 elements at a 128-byte stride}, box
// {64, 64, nblk}. One TMA instruction then fills nblk consecutive 8 KB swizzled
// blocks, which is the layout the UMMA MN-major descriptor expects.
int make_map_mn3(CUtensorMap* m, const void* base, bool bf16, uint64_t inner, uint64_t outer, uint64_t ld_elems,
                 uint32_t nblk) {
  if (reinterpret_cast<uintptr_t>(base) % 16 != 0) return fail(LMCE_ERR_INVALID_ARGUMENT, "tensor base not 16B aligned");
  if ((ld_elems * 2) % 16 != 0) return fail(LMCE_ERR_INVALID_ARGUMENT, "row stride not a multiple of 16 bytes");
  if (inner % 64 != 0) return fail(LMCE_ERR_INVALID_ARGUMENT, "3-D operand map needs a multiple of 64 columns");
  cuuint64_t dims[3] = {64, outer, inner / 64};
  cuuint64_t strides[2] = {ld_elems * 2, 128};
  cuuint32_t box[3] = {64, 64, nblk};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = g_encode(m, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3,
                        const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(LMCE_ERR_CUDA, "cuTensorMapEncodeTiled (3-D) failed (%d)", static_cast<int>(r));
  return LMCE_OK;
}

// Row-major 2-D fp32 tensor [outer][inner], box {box_inner, box_outer}, 128-byte swizzle
// (box_inner * 4 must be 128), for TMA stores and adds.
int make_map_f32(CUtensorMap* m, void* base, uint64_t inner, uint64_t outer, uint64_t ld_elems, uint32_t box_inner,
                 uint32_t box_outer) {
  if (reinterpret_cast<uintptr_t>(base) % 16 != 0) return fail(LMCE_ERR_INVALID_ARGUMENT, "tensor base not 16B aligned");
  if ((ld_elems * 4) % 16 != 0) return fail(LMCE_ERR_INVALID_ARGUMENT, "row stride not a multiple of 16 bytes");
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {ld_elems * 4};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, base, dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(LMCE_ERR_CUDA, "cuTensorMapEncodeTiled (fp32) failed (%d)", static_cast<int>(r));
  return LMCE_OK;
}

// A [outer][inner] tensor of 16-bit elements as the target of 32 x 32 TMA stores from a
// 64-byte-swizzled shared-memory box (the CTA-pair backward's dW epilogue).
int make_map_store16(CUtensorMap* m, void* base, bool bf16, uint64_t inner, uint64_t outer, uint64_t ld_elems) {
  if (reinterpret_cast<uintptr_t>(base) % 16 != 0) return fail(LMCE_ERR_INVALID_ARGUMENT, "tensor base not 16B aligned");
  if ((ld_elems * 2) % 16 != 0) return fail(LMCE_ERR_INVALID_ARGUMENT, "row stride not a multiple of 16 bytes");
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {ld_elems * 2};
  cuuint32_t box[2] = {32, 32};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode(m, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, base, dims,
                        strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(LMCE_ERR_CUDA, "cuTensorMapEncodeTiled (store) failed (%d)", static_cast<int>(r));
  return LMCE_OK;
}

// The same [outer][inner] tensor of 16-bit elements as a 3-D view {64 elements, outer,
// inner / 64 blocks at a 128-byte stride}, box {64, box_y, box_z}, 128-byte swizzle: a box
// reads box_z * 128 contiguous bytes of each of its box_y rows.
int make_map_3d(CUtensorMap* m, const void* base, bool bf16, uint64_t inner, uint64_t outer, uint64_t ld_elems,
                uint32_t box_y, uint32_t box_z) {
  if (reinterpret_cast<uintptr_t>(base) % 16 != 0) return fail(LMCE_ERR_INVALID_ARGUMENT, "tensor base not 16B aligned");
  if ((ld_elems * 2) % 16 != 0) return fail(LMCE_ERR_INVALID_ARGUMENT, "row stride not a multiple of 16 bytes");
  if (inner % 64 != 0) return fail(LMCE_ERR_INVALID_ARGUMENT, "3-D operand map needs a multiple of 64 columns");
  cuuint64_t dims[3] = {64, outer, inner / 64};
  cuuint64_t strides[2] = {ld_elems * 2, 128};
  cuuint32_t box[3] = {64, box_y, box_z};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = g_encode(m, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3,
                        const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(LMCE_ERR_CUDA, "cuTensorMapEncodeTiled (3-D) failed (%d)", static_cast<int>(r));
  return LMCE_OK;
}

// ---------------------------------------------------------------- engines ---

constexpr int kBN = BN;
constexpr int kStages = 4;

// Opt the kernel into its dynamic shared memory once per device.
template <typename K>
int ensure_smem_attr(K kern, int smem, bool* done) {
  int dev = 0;
  LMCE_CUDA(cudaGetDevice(&dev));
  if (!done[dev]) {
    LMCE_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    done[dev] = true;
  }
  return LMCE_OK;
}

// Launch with an optional cluster of 2 CTAs (pair kernels).
template <typename... KArgs, typename... Args>
int launch_ex(void (*kern)(KArgs...), int grid, int threads, int smem, int cluster, cudaStream_t st,
              Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid, 1, 1);
  cfg.blockDim = dim3(threads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = cluster;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
  if (e != cudaSuccess) return fail(LMCE_ERR_CUDA, "kernel launch failed: %s", cudaGetErrorString(e));
  return launched();
}

// Co-resident clusters of the pair kernel `kern` on the current device (cached per device and kernel).
template <typename K>
int max_pairs(K kern, int smem, int sms, int* cache, int threads = NUM_THREADS) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return sms / 2;
  if (cache[dev] > 0) return cache[dev];
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(sms, 1, 1);
  cfg.blockDim = dim3(threads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess || n <= 0) n = sms / 2;
  cache[dev] = n;
  return n;
}

template <bool BF16, bool PAIR>
int launch_stats(const CUtensorMap& mx, const CUtensorMap& mw, const StatsParams& p, int grid, cudaStream_t st) {
  auto kern = lmce_stats_kernel<BF16, PAIR>;
  constexpr int smem = TileCfg<PAIR>::SMEM_BYTES;
  static bool done[kMaxDevices] = {};
  if (int rc = ensure_smem_attr(kern, smem, done)) return rc;
  timing_mark(0, 0, st);
  const int rc = launch_ex(kern, grid, NUM_THREADS, smem, PAIR ? 2 : 1, st, mx, mw, p);
  timing_mark(0, 1, st);
  return rc;
}

// Statistics on CTA pairs for more than 128 tokens unless 256-row tiles add more than a
// quarter to the padded rows of 128-row ones: a pair's stage loads (one 256-byte-row box per
// operand, 64 bytes per clock of UMMA work at full rate) stay within what TMA delivers to an
// SM (~63 B/clk measured), a one-CTA 128 x 256 tile needs 96 B/clk and runs at ~2/3 of the
// tensor rate. LMCE_TILE_MODE (compile time): 0 = that rule, 1 = always single CTA, 2 = pairs
// where possible.
#ifndef LMCE_TILE_MODE
#define LMCE_TILE_MODE 0
#endif
bool use_pair_tiles(int64_t rows) {
  if (LMCE_TILE_MODE == 1) return false;
  if (LMCE_TILE_MODE == 2) return rows > BM;
  return rows > BM && ((rows + 255) / 256) * 256 * 4 <= ((rows + 127) / 128) * 128 * 5;
}

// Units that can run at once for the statistics kernel (CTAs, or pairs of CTAs).
int stats_slots(bool pair, int sms) {
  if (!pair) return sms;
  static int cache_f16[kMaxDevices] = {}, cache_bf16[kMaxDevices] = {};
  const int a = max_pairs(lmce_stats_kernel<false, true>, TileCfg<true>::SMEM_BYTES, sms, cache_f16);
  const int b = max_pairs(lmce_stats_kernel<true, true>, TileCfg<true>::SMEM_BYTES, sms, cache_bf16);
  return a < b ? a : b;
}

template <bool BF16>
int launch_bwd(const CUtensorMap* maps, const BwdParams& p, int grid, cudaStream_t st) {
  auto kern = lmce_bwd_kernel<BF16, kStages>;
  constexpr int smem = BWD_SMEM_BYTES;
  static bool done[kMaxDevices] = {};
  if (int rc = ensure_smem_attr(kern, smem, done)) return rc;
  timing_mark(1, 0, st);
  kern<<<grid, NUM_THREADS, smem, st>>>(maps[0], maps[1], maps[2], maps[3], maps[4], maps[5], p);
  const int rc = launched();
  timing_mark(1, 1, st);
  return rc;
}

// Backward on CTA pairs: one cluster of two per pair of SMs that can be co-resident.
template <bool BF16>
int launch_bwd_pair(const CUtensorMap* maps, const BwdParams& p, int sms, cudaStream_t st) {
  auto kern = lmce_bwd_pair_kernel<BF16>;
  constexpr int smem = PBWD_SMEM_BYTES;
  static bool done[kMaxDevices] = {};
  static int pairs_cache[kMaxDevices] = {};
  if (int rc = ensure_smem_attr(kern, smem, done)) return rc;
  const int pairs = max_pairs(kern, smem, sms, pairs_cache, P_THREADS);
  timing_mark(1, 0, st);
  const int rc = launch_ex(kern, 2 * pairs, P_THREADS, smem, 2, st, maps[0], maps[1], maps[2], maps[3], maps[4], p);
  timing_mark(1, 1, st);
  return rc;
}

// Which backward kernel runs: the CTA-pair kernel needs H >= 256 (3-D operand maps);
// LMCE_BWD_KERNEL=single forces the one-CTA kernel.
bool use_pair_backward(int64_t h) {
  static const int forced = [] {
    const char* e = std::getenv("LMCE_BWD_KERNEL");
    if (e && std::strcmp(e, "single") == 0) return 1;
    if (e && std::strcmp(e, "pair") == 0) return 2;
    return 0;
  }();
  if (h % 64 != 0 || h < kBN) return false;
  return forced != 1;
}

// Vocab slabs per token block: fill the SMs with whole waves of (block, slab)
// units while keeping slabs of near-equal tile counts.
int choose_slabs(int num_m, int num_n, int sms) {
  int best = 1;
  double best_eff = -1.0;
  const int smax = num_n < 256 ? num_n : 256;
  for (int s = 1; s <= smax; ++s) {
    const long long units = static_cast<long long>(num_m) * s;
    const long long waves = (units + sms - 1) / sms;
    const double fill = static_cast<double>(units) / static_cast<double>(waves * sms);
    const double per = static_cast<double>(num_n) / s;
    const double balance = per / static_cast<double>((num_n + s - 1) / s);
    const double eff = fill * balance;
    if (eff > best_eff + 1e-3) {
      best_eff = eff;
      best = s;
    }
  }
  return best;
}

// --------------------------------------------------------- aux kernels ---

__device__ __forceinline__ Part part_identity() {
  Part p;
  p.m = NEG_BIG;
  p.s = 0.f;
  p.w = 0.f;
  p.best = -INFINITY;
  p.idx = 0x7fffffff;
  p.zy = -INFINITY;
  return p;
}

__device__ __forceinline__ void part_merge(Part& a, const Part& b) {
  const float mx = fmaxf(a.m, b.m);
  const float da = a.m - mx, db = b.m - mx;
  const float ea = ex2_approx(da * LOG2E), eb = ex2_approx(db * LOG2E);
  const float s = a.s * ea + b.s * eb;
  const float w = ea * fmaf(da, a.s, a.w) + eb * fmaf(db, b.s, b.w);
  a.m = mx;
  a.s = s;
  a.w = w;
  if (b.best > a.best || (b.best == a.best && b.idx < a.idx)) {
    a.best = b.best;
    a.idx = b.idx;
  }
  a.zy = fmaxf(a.zy, b.zy);
}

__device__ __forceinline__ Part part_shfl_down(const Part& a, int off) {
  Part b;
  b.m = __shfl_down_sync(0xffffffffu, a.m, off);
  b.s = __shfl_down_sync(0xffffffffu, a.s, off);
  b.w = __shfl_down_sync(0xffffffffu, a.w, off);
  b.best = __shfl_down_sync(0xffffffffu, a.best, off);
  b.idx = __shfl_down_sync(0xffffffffu, a.idx, off);
  b.zy = __shfl_down_sync(0xffffffffu, a.zy, off);
  return b;
}

// One warp per token: lanes merge strided subsets of the records, then a
// fixed-shape shuffle tree (deterministic). FINAL=false writes the merged
// record; FINAL=true writes lse / nll / entropy / argmax.
template <bool FINAL>
__global__ void __launch_bounds__(256) stats_merge_kernel(const Part* __restrict__ parts, int n_parts,
                                                          long long tok_stride, long long part_stride,
                                                          int n_tokens, Part* __restrict__ rec_out,
                                                          const int64_t* __restrict__ labels,
                                                          float* __restrict__ lse_out, float* __restrict__ nll_out,
                                                          float* __restrict__ ent_out,
                                                          int64_t* __restrict__ arg_out, int* err) {
  const int lane = threadIdx.x & 31;
  const int warps_per_block = blockDim.x / 32;
  for (int t = blockIdx.x * warps_per_block + threadIdx.x / 32; t < n_tokens; t += gridDim.x * warps_per_block) {
    Part acc = part_identity();
    for (int pi = lane; pi < n_parts; pi += 32) {
      const Part* src = parts + static_cast<long long>(t) * tok_stride + static_cast<long long>(pi) * part_stride;
      const float2 a = reinterpret_cast<const float2*>(src)[0];
      const float2 b = reinterpret_cast<const float2*>(src)[1];
      const float2 c = reinterpret_cast<const float2*>(src)[2];
      Part q;
      q.m = a.x;
      q.s = a.y;
      q.w = b.x;
      q.best = b.y;
      q.idx = __float_as_int(c.x);
      q.zy = c.y;
      part_merge(acc, q);
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      const Part o = part_shfl_down(acc, off);
      part_merge(acc, o);
    }
    if (lane == 0) {
      if constexpr (!FINAL) {
        float2* d = reinterpret_cast<float2*>(rec_out + t);
        d[0] = make_float2(acc.m, acc.s);
        d[1] = make_float2(acc.w, acc.best);
        d[2] = make_float2(__int_as_float(acc.idx), acc.zy);
      } else {
        const float ln_s = lg2_approx(acc.s) * LN2;
        const float lse = acc.m + ln_s;
        const float ent = ln_s - acc.w / acc.s;
        const int64_t y = labels[t];
        float nll = 0.f;
        if (y != -100) {
          if (acc.zy == -INFINITY) {
            nll = __int_as_float(0x7fc00000);  // NaN: target outside [0, V)
            raise_error(err, ERR_LABEL);
          } else {
            nll = lse - acc.zy;
          }
        }
        lse_out[t] = lse;
        nll_out[t] = nll;
        ent_out[t] = ent;
        arg_out[t] = static_cast<int64_t>(acc.idx);
      }
    }
  }
}

// Deterministic loss: one block, fixed per-thread strided partial sums, fixed tree.
__global__ void __launch_bounds__(1024) loss_kernel(const float* __restrict__ nll, const int64_t* __restrict__ labels,
                                                    int n_tokens, const float* num_items_dev, float num_items,
                                                    float* loss, float* denom_out) {
  __shared__ float s_sum[32];
  __shared__ int s_cnt[32];
  float sum = 0.f;
  int cnt = 0;
  for (int t = threadIdx.x; t < n_tokens; t += blockDim.x) {
    sum += nll[t];
    cnt += labels[t] != -100 ? 1 : 0;
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    sum += __shfl_down_sync(0xffffffffu, sum, off);
    cnt += __shfl_down_sync(0xffffffffu, cnt, off);
  }
  const int w = threadIdx.x / 32;
  if ((threadIdx.x & 31) == 0) {
    s_sum[w] = sum;
    s_cnt[w] = cnt;
  }
  __syncthreads();
  if (w == 0) {
    const int nw = blockDim.x / 32;
    sum = threadIdx.x < nw ? s_sum[threadIdx.x] : 0.f;
    cnt = threadIdx.x < nw ? s_cnt[threadIdx.x] : 0;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      sum += __shfl_down_sync(0xffffffffu, sum, off);
      cnt += __shfl_down_sync(0xffffffffu, cnt, off);
    }
    if (threadIdx.x == 0) {
      // num_items NaN: not given (the count of labelled tokens); any other value is used as
      // given, then clamped to >= 1 like the reference's max(float(num_items_in_batch), 1.0)
      float d = num_items_dev ? *num_items_dev : (isnan(num_items) ? static_cast<float>(cnt) : num_items);
      d = fmaxf(d, 1.0f);
      *denom_out = d;
      *loss = sum / d;
    }
  }
}

// Stable compaction of tokens with label != -100 (one block).
__global__ void __launch_bounds__(1024) compact_kernel(const int64_t* __restrict__ labels, int n_tokens,
                                                       long long v_off, int v_local, const float* __restrict__ lse,
                                                       int* __restrict__ count, int* __restrict__ row_idx,
                                                       int* __restrict__ lbl_lab, float* __restrict__ lse_lab) {
  __shared__ int s_warp[32];
  const int per = (n_tokens + blockDim.x - 1) / blockDim.x;
  const int t0 = threadIdx.x * per;
  const int t1 = min(t0 + per, n_tokens);
  int c = 0;
  for (int t = t0; t < t1; ++t) c += labels[t] != -100 ? 1 : 0;
  // block exclusive scan of c
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
    const int nw = blockDim.x / 32;
    int v = lane < nw ? s_warp[lane] : 0;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int o = __shfl_up_sync(0xffffffffu, v, off);
      if (lane >= off) v += o;
    }
    if (lane < nw) s_warp[lane] = v;  // inclusive warp totals
  }
  __syncthreads();
  int pos = incl - c + (w > 0 ? s_warp[w - 1] : 0);
  for (int t = t0; t < t1; ++t) {
    const int64_t y = labels[t];
    if (y != -100) {
      const long long yl = y - v_off;
      row_idx[pos] = t;
      lbl_lab[pos] = (yl >= 0 && yl < v_local) ? static_cast<int>(yl) : -1;
      lse_lab[pos] = lse[t];
      ++pos;
    }
  }
  if (threadIdx.x == blockDim.x - 1) *count = pos;
}

// X_lab[r] = X[row_idx[r]] for r < count, zero rows for count <= r < rows_pad. 16-byte vectors.
__global__ void gather_rows_kernel(const uint4* __restrict__ x, int vec_per_row, const int* __restrict__ count,
                                   const int* __restrict__ row_idx, int rows_pad, uint4* __restrict__ out) {
  const int n = *count;
  const long long total = static_cast<long long>(rows_pad) * vec_per_row;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int r = static_cast<int>(i / vec_per_row);
    const int c = static_cast<int>(i % vec_per_row);
    uint4 v = make_uint4(0, 0, 0, 0);
    if (r < n) v = x[static_cast<long long>(row_idx[r]) * vec_per_row + c];
    out[i] = v;
  }
}

template <bool BF16>
__global__ void dx_finalize_kernel(const float4* __restrict__ src, long long n4, uint2* __restrict__ dst) {
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n4;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const float4 v = src[i];
    uint2 o;
    o.x = pack2<BF16>(v.x, v.y);
    o.y = pack2<BF16>(v.z, v.w);
    dst[i] = o;
  }
}

// dst row t = src row t for labelled tokens, zeros otherwise (rows of `vec` 16-byte units).
__global__ void dx_copy_labelled_kernel(const uint4* __restrict__ src, const int64_t* __restrict__ labels, int vec,
                                        long long total, uint4* __restrict__ dst) {
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long t = i / vec;
    dst[i] = labels[t] != -100 ? src[i] : make_uint4(0u, 0u, 0u, 0u);
  }
}

__global__ void selftest_wait_kernel(unsigned long long timeout_ns, int* err) {
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    // Nothing ever arrives on `bar`: the bounded wait must give up.
    if (!mbar_wait(&bar, 0, &abort_flag, timeout_ns)) raise_error(err, ERR_TIMEOUT);
    // Complete the phase so the barrier is left in a clean state.
    mbar_arrive(&bar);
  }
  __syncthreads();
}

// TMA pipeline probe (diagnostic): one CTA per SM streams `iters` stages from a tensor through
// a ring of `stages` stages of `stage_bytes`; one thread loads each stage as soon as it is
// free, another waits for it, holds it `hold` cycles (a stand-in for the UMMAs that read a
// stage) and frees it. kind 0: 2-D {64, 128} boxes (128 bytes of each of 128 rows, 16 KB);
// kind 1: 3-D {64, 128, 2} boxes (256 contiguous bytes of each of 128 rows, 32 KB), the boxes
// the kernels load; kind 2: plain bulk copies of 32 contiguous KB. Every wait is bounded.
constexpr int PROBE_MAX_STAGES = 8;
constexpr int PROBE_MAX_SMEM = 226 * 1024;  // dynamic, below the 227 KB opt-in limit
__global__ void __launch_bounds__(64, 1) tma_pipeline_probe_kernel(
    const __grid_constant__ CUtensorMap map2, const __grid_constant__ CUtensorMap map3, const uint8_t* base,
    long long n_pieces32, int kind, int stage_bytes, int stages, int hold, int iters, int row_blocks, int kblocks,
    unsigned long long timeout_ns, unsigned long long* cycles, int* err) {
  extern __shared__ uint8_t raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + static_cast<size_t>(stages) * stage_bytes);
  uint64_t* empty = full + PROBE_MAX_STAGES;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();
  const int piece = kind == 0 ? 16384 : 32768;
  const int pieces = stage_bytes / piece;
  if (threadIdx.x == 0) {
    int stage = 0;
    uint32_t phase = 0;
    for (int i = 0; i < iters; ++i) {
      if (!mbar_wait(&empty[stage], phase ^ 1u, &abort_flag, timeout_ns)) {
        raise_error(err, ERR_TIMEOUT);
        abort_flag = 1;
        break;
      }
      mbar_arrive_expect_tx(&full[stage], static_cast<uint32_t>(stage_bytes));
      uint8_t* dst = smem + static_cast<size_t>(stage) * stage_bytes;
      for (int q = 0; q < pieces; ++q) {
        const long long u = static_cast<long long>(blockIdx.x) * 7919 + static_cast<long long>(i) * pieces + q;
        if (kind == 0) {  // one 64-element block of one 128-row block
          tma_load_2d(dst + q * piece, &map2, &full[stage], static_cast<int>(u % kblocks) * 64,
                      static_cast<int>((u / kblocks) % row_blocks) * 128);
        } else if (kind == 1) {  // two adjacent 64-element blocks of one 128-row block
          const int kp = kblocks / 2;
          tma_load_3d(dst + q * piece, &map3, &full[stage], 0, static_cast<int>((u / kp) % row_blocks) * 128,
                      static_cast<int>(u % kp) * 2);
        } else {
          bulk_load(dst + q * piece, base + (u % n_pieces32) * 32768, 32768, &full[stage]);
        }
      }
      if (++stage == stages) {
        stage = 0;
        phase ^= 1u;
      }
    }
  } else if (threadIdx.x == 32) {
    int stage = 0;
    uint32_t phase = 0;
    long long t0 = 0, t1 = 0;
    for (int i = 0; i < iters; ++i) {
      if (!mbar_wait(&full[stage], phase, &abort_flag, timeout_ns)) {
        raise_error(err, ERR_TIMEOUT);
        abort_flag = 1;
        break;
      }
      const long long got = clock64();
      if (i == 8) t0 = got;
      while (clock64() - got < hold) {
      }
      if (i == iters - 1) t1 = clock64();
      mbar_arrive(&empty[stage]);
      if (++stage == stages) {
        stage = 0;
        phase ^= 1u;
      }
    }
    cycles[blockIdx.x] = static_cast<unsigned long long>(t1 - t0);
  }
  __syncthreads();
}

// ------------------------------------------------------------ workspace ---

size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

struct BwdLayout {
  size_t count, row_idx, lbl_lab, lse_lab, x_lab, g, dx_acc, sync, total;
  int rows_pad, v_chunk, n_chunks, sync_ints;
};

// Default vocab chunk of the backward. CTA-pair kernel: gradient buffers (three of
// rows_pad x v_chunk) of about 90 MiB, within 4096..20480 vocab rows; measured on one B200
// at config 2 under sustained load, 8192-row chunks run within 0.3% of 20480-row ones (the
// K = 128 stages keep the UMMA fed at every chunk width), so the memory-lean size is the
// default. One-CTA kernel: about 64 MiB within 8192..32768 rows. For few tokens the chunk
// is also capped so that the G buffers stay at most half the size of an [N, V] logits
// buffer: with the 256-row padding of the [rows, H] buffers the whole workspace stays
// below [N, V] in the input dtype for every N >= 64.
int64_t auto_v_chunk(int64_t n, int64_t rows_pad, int64_t v_local, bool pair) {
  int64_t vc;
  if (pair) {
    vc = (90ll << 20) / (2 * NUM_GBUF * rows_pad) / 256 * 256;
    if (vc < 4096) vc = 4096;
    if (vc > 20480) vc = 20480;
  } else {
    vc = (64ll << 20) / (2 * rows_pad) / 2048 * 2048;
    if (vc < 8192) vc = 8192;
    if (vc > 32768) vc = 32768;
  }
  const int64_t g_rows = NUM_GBUF * ((n + 255) / 256 * 256);
  const int64_t cap = (n * v_local / 2) / g_rows / 256 * 256;  // G bytes <= n * v_local bytes
  if (vc > cap) vc = cap < 256 ? 256 : cap;
  return vc;
}

BwdLayout bwd_layout(int64_t n, int64_t h, int64_t v_local, int64_t v_chunk) {
  BwdLayout L{};
  const int64_t rows_pad = (n + BM - 1) / BM * BM;
  int64_t vc = v_chunk <= 0 ? auto_v_chunk(n, rows_pad, v_local, use_pair_backward(h)) : v_chunk;
  vc = (vc + 255) / 256 * 256;
  const int64_t vmax = (v_local + 255) / 256 * 256;
  if (vc > vmax) vc = vmax;
  if (vc < 256) vc = 256;
  L.v_chunk = static_cast<int>(vc);
  L.n_chunks = static_cast<int>((v_local + vc - 1) / vc);
  L.rows_pad = static_cast<int>((n + 255) / 256 * 256);  // row blocks of 256 (pair kernel), 128 (one-CTA)
  const int num_hn = static_cast<int>((h + BN - 1) / BN);
  L.sync_ints = 1 + 2 * L.n_chunks + (L.rows_pad / BM) * num_hn + 1;
  size_t off = 0;
  L.count = off;
  off = align_up(off + 16, 256);
  L.row_idx = off;
  off = align_up(off + sizeof(int) * n, 256);
  L.lbl_lab = off;
  off = align_up(off + sizeof(int) * n, 256);
  L.lse_lab = off;
  off = align_up(off + sizeof(float) * n, 256);
  L.x_lab = off;
  off = align_up(off + 2ull * L.rows_pad * h, 256);
  L.g = off;
  off = align_up(off + 2ull * NUM_GBUF * L.rows_pad * vc, 256);
  L.dx_acc = off;
  off = align_up(off + 4ull * L.rows_pad * h, 256);
  L.sync = off;
  off = align_up(off + sizeof(int) * L.sync_ints, 256);
  L.total = off;
  return L;
}

bool aligned16(const void* p) { return reinterpret_cast<uintptr_t>(p) % 16 == 0; }

}  // namespace

// =================================================================== C ABI ===

extern "C" {

int lmce_abi_version(void) { return LMCE_ABI_VERSION; }

const char* lmce_last_error(void) { return t_err; }

int lmce_device_error(int reset) {
  DevInfo* d = nullptr;
  if (int rc = device_info(&d)) return rc;
  int v = 0;
  LMCE_CUDA(cudaMemcpy(&v, d->err_ptr, sizeof(int), cudaMemcpyDeviceToHost));
  if (reset) {
    const int z = 0;
    LMCE_CUDA(cudaMemcpy(d->err_ptr, &z, sizeof(int), cudaMemcpyHostToDevice));
  }
  if (v != 0) fail(v, "device error word = %d", v);
  return v;
}

int64_t lmce_fwd_num_parts(int64_t n_tokens, int64_t vocab_local) {
  DevInfo* d = nullptr;
  int sms = 148;
  if (device_info(&d) == LMCE_OK) sms = d->sms;
  if (n_tokens <= 0 || vocab_local <= 0) return 1;
  const bool pair = use_pair_tiles(n_tokens);
  const int tile_m = pair ? 2 * BM : BM;
  const int num_m = static_cast<int>((n_tokens + tile_m - 1) / tile_m);
  const int num_n = static_cast<int>((vocab_local + kBN - 1) / kBN);
  return choose_slabs(num_m, num_n, d ? stats_slots(pair, sms) : sms);
}

int lmce_fwd_stats(const void* hidden, const void* weight, const int64_t* labels, int64_t n_tokens,
                   int64_t hidden_dim, int64_t vocab_local, int64_t vocab_offset, int dtype, lmce_part* parts,
                   int64_t n_parts, void* stream) {
  if (!hidden || !weight || !labels || !parts) return fail(LMCE_ERR_INVALID_ARGUMENT, "null pointer");
  if (n_tokens <= 0 || n_tokens > (1ll << 30)) return fail(LMCE_ERR_INVALID_ARGUMENT, "bad n_tokens %lld", (long long)n_tokens);
  if (vocab_local <= 0 || vocab_local + vocab_offset > (1ll << 31) - 1 || vocab_offset < 0)
    return fail(LMCE_ERR_INVALID_ARGUMENT, "bad vocab size/offset");
  if (hidden_dim <= 0 || hidden_dim % 64 != 0) return fail(LMCE_ERR_UNSUPPORTED, "hidden_dim must be a positive multiple of 64");
  if (dtype != LMCE_DTYPE_F16 && dtype != LMCE_DTYPE_BF16) return fail(LMCE_ERR_UNSUPPORTED, "dtype %d", dtype);
  DevInfo* d = nullptr;
  if (int rc = device_info(&d)) return rc;
  if (int rc = get_encoder()) return rc;
  const bool pair = use_pair_tiles(n_tokens);
  const int tile_m = pair ? 2 * BM : BM;
  const int num_m = static_cast<int>((n_tokens + tile_m - 1) / tile_m);
  const int num_n = static_cast<int>((vocab_local + kBN - 1) / kBN);
  if (n_parts < 1 || n_parts > num_n) return fail(LMCE_ERR_INVALID_ARGUMENT, "n_parts %lld out of range", (long long)n_parts);
  const bool bf16 = dtype == LMCE_DTYPE_BF16;
  CUtensorMap mx, mw;
  if (pair) {  // 3-D views, box {64, 128, 2}: a CTA's 128 rows x two k-blocks per stage
    if (int rc = make_map_3d(&mx, hidden, bf16, hidden_dim, n_tokens, hidden_dim, 128, 2)) return rc;
    if (int rc = make_map_3d(&mw, weight, bf16, hidden_dim, vocab_local, hidden_dim, 128, 2)) return rc;
  } else {
    if (int rc = make_map(&mx, hidden, bf16, hidden_dim, n_tokens, hidden_dim, BM)) return rc;
    if (int rc = make_map(&mw, weight, bf16, hidden_dim, vocab_local, hidden_dim, kBN)) return rc;
  }
  StatsParams p{};
  p.M = static_cast<int>(n_tokens);
  p.N = static_cast<int>(vocab_local);
  p.K = static_cast<int>(hidden_dim);
  p.n_slabs = static_cast<int>(n_parts);
  p.labels = labels;
  p.label_off = vocab_offset;
  p.parts = reinterpret_cast<Part*>(parts);
  p.err = d->err_ptr;
  p.timeout_ns = wait_timeout_ns();
  const long long units = static_cast<long long>(num_m) * n_parts;
  const int slots = stats_slots(pair, d->sms);
  const int grid = static_cast<int>(units < slots ? units : slots) * (pair ? 2 : 1);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (pair)
    return bf16 ? launch_stats<true, true>(mx, mw, p, grid, st) : launch_stats<false, true>(mx, mw, p, grid, st);
  return bf16 ? launch_stats<true, false>(mx, mw, p, grid, st) : launch_stats<false, false>(mx, mw, p, grid, st);
}

int lmce_stats_reduce(const lmce_part* parts, int64_t n_parts, int64_t tok_stride, int64_t part_stride,
                      int64_t n_tokens, lmce_part* record_out, void* stream) {
  if (!parts || !record_out || n_parts < 1 || n_tokens < 1) return fail(LMCE_ERR_INVALID_ARGUMENT, "bad arguments");
  DevInfo* d = nullptr;
  if (int rc = device_info(&d)) return rc;
  const int warps = 8;
  long long blocks = (n_tokens + warps - 1) / warps;
  if (blocks > 65535ll * 4) blocks = 65535ll * 4;
  stats_merge_kernel<false><<<static_cast<int>(blocks), warps * 32, 0, static_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const Part*>(parts), static_cast<int>(n_parts), tok_stride, part_stride,
      static_cast<int>(n_tokens), reinterpret_cast<Part*>(record_out), nullptr, nullptr, nullptr, nullptr, nullptr,
      d->err_ptr);
  return launched();
}

int lmce_stats_finish(const lmce_part* parts, int64_t n_parts, int64_t tok_stride, int64_t part_stride,
                      const int64_t* labels, int64_t n_tokens, const float* num_items_dev, double num_items,
                      float* lse, float* nll, float* entropy, int64_t* argmax, float* loss, float* denom,
                      void* stream) {
  if (!parts || !labels || !lse || !nll || !entropy || !argmax || !loss || !denom || n_parts < 1 || n_tokens < 1)
    return fail(LMCE_ERR_INVALID_ARGUMENT, "bad arguments");
  DevInfo* d = nullptr;
  if (int rc = device_info(&d)) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int warps = 8;
  long long blocks = (n_tokens + warps - 1) / warps;
  if (blocks > 65535ll * 4) blocks = 65535ll * 4;
  stats_merge_kernel<true><<<static_cast<int>(blocks), warps * 32, 0, st>>>(
      reinterpret_cast<const Part*>(parts), static_cast<int>(n_parts), tok_stride, part_stride,
      static_cast<int>(n_tokens), nullptr, labels, lse, nll, entropy, argmax, d->err_ptr);
  if (int rc = launched()) return rc;
  loss_kernel<<<1, 1024, 0, st>>>(nll, labels, static_cast<int>(n_tokens), num_items_dev,
                                  static_cast<float>(num_items), loss, denom);
  return launched();
}

size_t lmce_bwd_workspace_bytes(int64_t n_tokens, int64_t hidden_dim, int64_t vocab_local, int64_t v_chunk) {
  if (n_tokens <= 0 || hidden_dim <= 0 || vocab_local <= 0) return 0;
  return bwd_layout(n_tokens, hidden_dim, vocab_local, v_chunk).total;
}

}  // extern "C"

namespace {

int backward_impl(const void* hidden, const void* weight, const int64_t* labels, const float* lse, int64_t n_tokens,
                  int64_t hidden_dim, int64_t vocab_local, int64_t vocab_offset, int dtype, const float* grad_loss,
                  const float* denom, void* d_hidden, float* d_hidden_f32, const lmce_dx_exchange* xch, void* d_weight,
                  int64_t v_chunk, void* workspace, size_t workspace_bytes, void* stream) {
  if (!hidden || !weight || !labels || !lse || !denom || !workspace)
    return fail(LMCE_ERR_INVALID_ARGUMENT, "null pointer");
  if (n_tokens <= 0 || n_tokens > (1ll << 30)) return fail(LMCE_ERR_INVALID_ARGUMENT, "bad n_tokens");
  if (vocab_local <= 0 || vocab_offset < 0 || vocab_local + vocab_offset > (1ll << 31) - 1)
    return fail(LMCE_ERR_INVALID_ARGUMENT, "bad vocab size/offset");
  if (hidden_dim <= 0 || hidden_dim % 64 != 0) return fail(LMCE_ERR_UNSUPPORTED, "hidden_dim must be a positive multiple of 64");
  if (dtype != LMCE_DTYPE_F16 && dtype != LMCE_DTYPE_BF16) return fail(LMCE_ERR_UNSUPPORTED, "dtype %d", dtype);
  if ((d_hidden && !aligned16(d_hidden)) || (d_hidden_f32 && !aligned16(d_hidden_f32)) ||
      (xch && (!aligned16(xch->partial) || !aligned16(xch->partial_mc) || !aligned16(xch->out_mc))) ||
      (d_weight && !aligned16(d_weight)) || !aligned16(workspace))
    return fail(LMCE_ERR_INVALID_ARGUMENT, "output/workspace buffers must be 16-byte aligned");
  if (xch && (!xch->partial || !xch->partial_mc || !xch->out_mc || !xch->flags || !xch->flags_mc ||
              xch->world < 1 || xch->rank < 0 || xch->rank >= xch->world || xch->epoch == 0))
    return fail(LMCE_ERR_INVALID_ARGUMENT, "bad dX exchange buffers");
  const BwdLayout L = bwd_layout(n_tokens, hidden_dim, vocab_local, v_chunk);
  if (workspace_bytes < L.total)
    return fail(LMCE_ERR_WORKSPACE, "workspace %zu bytes < required %zu", workspace_bytes, L.total);
  DevInfo* d = nullptr;
  if (int rc = device_info(&d)) return rc;
  if (int rc = get_encoder()) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const bool bf16 = dtype == LMCE_DTYPE_BF16;
  const int n = static_cast<int>(n_tokens), h = static_cast<int>(hidden_dim), vl = static_cast<int>(vocab_local);
  char* ws = static_cast<char*>(workspace);
  int* count = reinterpret_cast<int*>(ws + L.count);
  int* row_idx = reinterpret_cast<int*>(ws + L.row_idx);
  int* lbl_lab = reinterpret_cast<int*>(ws + L.lbl_lab);
  float* lse_lab = reinterpret_cast<float*>(ws + L.lse_lab);
  void* x_lab = ws + L.x_lab;
  void* g = ws + L.g;
  float* dx_acc = reinterpret_cast<float*>(ws + L.dx_acc);

  if (d_hidden) LMCE_CUDA(cudaMemsetAsync(d_hidden, 0, 2ull * n * h, st));

  compact_kernel<<<1, 1024, 0, st>>>(labels, n, vocab_offset, vl, lse, count, row_idx, lbl_lab, lse_lab);
  if (int rc = launched()) return rc;
  {
    const int vec = h * 2 / 16;
    const long long total = static_cast<long long>(L.rows_pad) * vec;
    long long blocks = (total + 255) / 256;
    if (blocks > d->sms * 8ll) blocks = d->sms * 8ll;
    gather_rows_kernel<<<static_cast<int>(blocks), 256, 0, st>>>(static_cast<const uint4*>(hidden), vec, count,
                                                                 row_idx, L.rows_pad, static_cast<uint4*>(x_lab));
    if (int rc = launched()) return rc;
  }

  if (xch) d_hidden_f32 = xch->partial;
  const bool want_dx = d_hidden != nullptr || d_hidden_f32 != nullptr;
  const bool want_dw = d_weight != nullptr;
  if (!want_dx && !want_dw) return LMCE_OK;

  // Tensor maps (tile offsets are TMA coordinates). MN-major operands load through 3-D
  // maps (one TMA instruction per operand and k-block instead of one per 64 columns; the
  // producer thread's issue rate bounds the DX and DW tiles otherwise). The three G
  // buffers are one tensor: for the CTA-pair kernel G^T [NUM_GBUF * v_chunk, rows_pad]
  // (buffer b starts at vocab row b * v_chunk), for the one-CTA kernel G
  // [NUM_GBUF * rows_pad, v_chunk] (buffer b starts at token row b * rows_pad).
  CUtensorMap maps[7];
  std::memset(maps, 0, sizeof(maps));
  const int g_rows = NUM_GBUF * L.rows_pad;
  const int gt_rows = NUM_GBUF * L.v_chunk;
  const bool pair = use_pair_backward(h);
  const bool mn3_h = h % 64 == 0 && h >= kBN;
  if (pair) {
    // W [V][H], X_lab [rows_pad][H] and G^T [NUM_GBUF * v_chunk][rows_pad], each as a 3-D view
    // {64 elements, rows, 64-element blocks} with box {64, 128, 2}: one box is a CTA's share of
    // a stage, K-major (128 rows x two k-blocks) or MN-major (128 k-rows x two MN blocks) alike
    if (int rc = make_map_3d(&maps[0], weight, bf16, h, vl, h, 128, 2)) return rc;
    if (int rc = make_map_3d(&maps[1], x_lab, bf16, h, L.rows_pad, h, 128, 2)) return rc;
    if (int rc = make_map_3d(&maps[2], g, bf16, L.rows_pad, gt_rows, L.rows_pad, 128, 2)) return rc;
    // the fp32 dX^T accumulator [H][rows_pad], 32 x 32 boxes for the epilogue's TMA stores and adds
    if (int rc = make_map_f32(&maps[3], dx_acc, L.rows_pad, h, L.rows_pad, 32, 32)) return rc;
    // dW [V][H]: 32 x 32 boxes for the epilogue's TMA stores
    if (d_weight != nullptr)
      if (int rc = make_map_store16(&maps[4], d_weight, bf16, h, vl, h)) return rc;
  } else {
    // x K-major, x MN-major, W K-major, W MN-major, G K-major, G MN-major (X and W fall
    // back to 2-D MN-major maps when H is below 256)
    if (int rc = make_map(&maps[0], x_lab, bf16, h, L.rows_pad, h, BM)) return rc;
    if (int rc = mn3_h ? make_map_mn3(&maps[1], x_lab, bf16, h, L.rows_pad, h, kBN / 64)
                       : make_map(&maps[1], x_lab, bf16, h, L.rows_pad, h, 64))
      return rc;
    if (int rc = make_map(&maps[2], weight, bf16, h, vl, h, kBN)) return rc;
    if (int rc = mn3_h ? make_map_mn3(&maps[3], weight, bf16, h, vl, h, kBN / 64)
                       : make_map(&maps[3], weight, bf16, h, vl, h, 64))
      return rc;
    if (int rc = make_map(&maps[4], g, bf16, L.v_chunk, g_rows, L.v_chunk, BM)) return rc;
    if (int rc = make_map_mn3(&maps[5], g, bf16, L.v_chunk, g_rows, L.v_chunk, BM / 64)) return rc;
  }

  int* sync = reinterpret_cast<int*>(ws + L.sync);
  LMCE_CUDA(cudaMemsetAsync(sync, 0, sizeof(int) * L.sync_ints, st));

  BwdParams p{};
  p.rows_pad = L.rows_pad;
  p.H = h;
  p.V = vl;
  p.v_chunk = L.v_chunk;
  p.n_chunks = L.n_chunks;
  p.count = count;
  p.lbl_lab = lbl_lab;
  p.lse_lab = lse_lab;
  p.g = g;
  p.dx_acc = dx_acc;
  p.row_idx = row_idx;
  p.dx_out = d_hidden;
  p.dx_out_f32 = d_hidden_f32;
  if (xch) {
    // rank r sums columns [x_lo, x_hi) of every row block (8-column groups split evenly)
    const int groups = h / 8;
    p.x_part_mc = xch->partial_mc;
    p.x_out_mc = xch->out_mc;
    p.x_flags = xch->flags;
    p.x_flags_mc = xch->flags_mc;
    p.x_epoch = xch->epoch;
    p.x_rank = xch->rank;
    p.x_world = xch->world;
    p.x_lo = groups * xch->rank / xch->world * 8;
    p.x_hi = groups * (xch->rank + 1) / xch->world * 8;
  }
  p.dw_out = d_weight;
  p.want_dx = want_dx ? 1 : 0;
  p.want_dw = want_dw ? 1 : 0;
  p.mn3_h = mn3_h ? 1 : 0;
  p.grad_loss = grad_loss;
  p.denom = denom;
  p.gscale = GSCALE;
  p.sync = sync;
  p.err = d->err_ptr;
  p.timeout_ns = wait_timeout_ns();
  const int grid = d->sms;
  if (pair) return bf16 ? launch_bwd_pair<true>(maps, p, grid, st) : launch_bwd_pair<false>(maps, p, grid, st);
  return bf16 ? launch_bwd<true>(maps, p, grid, st) : launch_bwd<false>(maps, p, grid, st);
}

}  // namespace

extern "C" {

int lmce_backward(const void* hidden, const void* weight, const int64_t* labels, const float* lse,
                  int64_t n_tokens, int64_t hidden_dim, int64_t vocab_local, int64_t vocab_offset, int dtype,
                  const float* grad_loss, const float* denom, void* d_hidden, float* d_hidden_f32,
                  void* d_weight, int64_t v_chunk, void* workspace, size_t workspace_bytes, void* stream) {
  return backward_impl(hidden, weight, labels, lse, n_tokens, hidden_dim, vocab_local, vocab_offset, dtype, grad_loss,
                       denom, d_hidden, d_hidden_f32, nullptr, d_weight, v_chunk, workspace, workspace_bytes, stream);
}

int lmce_backward_nvls(const void* hidden, const void* weight, const int64_t* labels, const float* lse,
                       int64_t n_tokens, int64_t hidden_dim, int64_t vocab_local, int64_t vocab_offset, int dtype,
                       const float* grad_loss, const float* denom, const lmce_dx_exchange* xch, void* d_weight,
                       int64_t v_chunk, void* workspace, size_t workspace_bytes, void* stream) {
  if (xch == nullptr) return fail(LMCE_ERR_INVALID_ARGUMENT, "null dX exchange descriptor");
  return backward_impl(hidden, weight, labels, lse, n_tokens, hidden_dim, vocab_local, vocab_offset, dtype, grad_loss,
                       denom, nullptr, nullptr, xch, d_weight, v_chunk, workspace, workspace_bytes, stream);
}

int lmce_dx_finalize(const float* d_hidden_f32, int64_t n_tokens, int64_t hidden_dim, int dtype, void* d_hidden,
                     void* stream) {
  if (!d_hidden_f32 || !d_hidden || n_tokens <= 0 || hidden_dim <= 0 || hidden_dim % 4 != 0)
    return fail(LMCE_ERR_INVALID_ARGUMENT, "bad arguments");
  if (!aligned16(d_hidden_f32) || reinterpret_cast<uintptr_t>(d_hidden) % 8 != 0)
    return fail(LMCE_ERR_INVALID_ARGUMENT, "misaligned buffers");
  DevInfo* d = nullptr;
  if (int rc = device_info(&d)) return rc;
  const long long n4 = n_tokens * hidden_dim / 4;
  long long blocks = (n4 + 255) / 256;
  if (blocks > d->sms * 8ll) blocks = d->sms * 8ll;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (dtype == LMCE_DTYPE_BF16)
    dx_finalize_kernel<true><<<static_cast<int>(blocks), 256, 0, st>>>(reinterpret_cast<const float4*>(d_hidden_f32),
                                                                       n4, static_cast<uint2*>(d_hidden));
  else if (dtype == LMCE_DTYPE_F16)
    dx_finalize_kernel<false><<<static_cast<int>(blocks), 256, 0, st>>>(
        reinterpret_cast<const float4*>(d_hidden_f32), n4, static_cast<uint2*>(d_hidden));
  else
    return fail(LMCE_ERR_UNSUPPORTED, "dtype %d", dtype);
  return launched();
}

int lmce_dx_copy_labelled(const void* src, const int64_t* labels, int64_t n_tokens, int64_t hidden_dim, int dtype,
                          void* d_hidden, void* stream) {
  if (!src || !labels || !d_hidden || n_tokens <= 0 || hidden_dim <= 0 || hidden_dim % 8 != 0)
    return fail(LMCE_ERR_INVALID_ARGUMENT, "bad arguments");
  if (dtype != LMCE_DTYPE_F16 && dtype != LMCE_DTYPE_BF16) return fail(LMCE_ERR_UNSUPPORTED, "dtype %d", dtype);
  if (!aligned16(src) || !aligned16(d_hidden)) return fail(LMCE_ERR_INVALID_ARGUMENT, "misaligned buffers");
  DevInfo* d = nullptr;
  if (int rc = device_info(&d)) return rc;
  const int vec = static_cast<int>(hidden_dim * 2 / 16);
  const long long total = n_tokens * vec;
  long long blocks = (total + 255) / 256;
  if (blocks > d->sms * 8ll) blocks = d->sms * 8ll;
  dx_copy_labelled_kernel<<<static_cast<int>(blocks), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint4*>(src), labels, vec, total, static_cast<uint4*>(d_hidden));
  return launched();
}

int lmce_pack_tokens(const int64_t* labels, const int64_t* attention_mask, int64_t batch, int64_t seq,
                     int64_t* shift_labels, int64_t* valid_idx, int32_t* row_lengths, int32_t* count,
                     const void* hidden, int64_t hidden_dim, int dtype, void* hidden_packed, void* stream) {
  if (!labels || !shift_labels || !valid_idx || !row_lengths || !count)
    return fail(LMCE_ERR_INVALID_ARGUMENT, "null pointer");
  if (batch <= 0 || seq <= 0 || batch * seq > (1ll << 22))
    return fail(LMCE_ERR_INVALID_ARGUMENT, "bad batch/seq (1 <= B*S <= 2^22)");
  if ((hidden == nullptr) != (hidden_packed == nullptr))
    return fail(LMCE_ERR_INVALID_ARGUMENT, "hidden and hidden_packed go together");
  if (hidden) {
    if (hidden_dim <= 0 || hidden_dim % 8 != 0) return fail(LMCE_ERR_INVALID_ARGUMENT, "hidden_dim must be a multiple of 8");
    if (dtype != LMCE_DTYPE_F16 && dtype != LMCE_DTYPE_BF16) return fail(LMCE_ERR_UNSUPPORTED, "dtype %d", dtype);
    if (!aligned16(hidden) || !aligned16(hidden_packed)) return fail(LMCE_ERR_INVALID_ARGUMENT, "misaligned buffers");
  }
  DevInfo* d = nullptr;
  if (int rc = device_info(&d)) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  LMCE_CUDA(cudaMemsetAsync(row_lengths, 0, sizeof(int32_t) * batch, st));
  pack_tokens_kernel<<<1, PACK_THREADS, 0, st>>>(labels, attention_mask, batch, seq, shift_labels, valid_idx,
                                                 row_lengths, count);
  if (int rc = launched()) return rc;
  if (!hidden) return LMCE_OK;
  const int vec = static_cast<int>(hidden_dim * 2 / 16);
  long long blocks = (batch * seq * vec + 255) / 256;
  if (blocks > d->sms * 8ll) blocks = d->sms * 8ll;
  pack_rows_kernel<<<static_cast<int>(blocks), 256, 0, st>>>(static_cast<const uint4*>(hidden), vec, valid_idx,
                                                             count, static_cast<uint4*>(hidden_packed));
  return launched();
}

int lmce_scatter_token_outputs(const float* nll, const float* entropy, const int64_t* argmax,
                               const int64_t* valid_idx, const int32_t* count, int64_t total, float* full_nll,
                               float* full_entropy, int64_t* full_argmax, void* stream) {
  if (!nll || !entropy || !argmax || !valid_idx || !count || !full_nll || !full_entropy || !full_argmax)
    return fail(LMCE_ERR_INVALID_ARGUMENT, "null pointer");
  if (total <= 0 || total > (1ll << 22)) return fail(LMCE_ERR_INVALID_ARGUMENT, "bad total (1 <= total <= 2^22)");
  DevInfo* d = nullptr;
  if (int rc = device_info(&d)) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  fill_outputs_kernel<<<1, PACK_THREADS, 0, st>>>(entropy, count, total, full_nll, full_entropy, full_argmax);
  if (int rc = launched()) return rc;
  long long blocks = (total + 255) / 256;
  if (blocks > d->sms * 4ll) blocks = d->sms * 4ll;
  scatter_outputs_kernel<<<static_cast<int>(blocks), 256, 0, st>>>(nll, entropy, argmax, valid_idx, count, full_nll,
                                                                   full_entropy, full_argmax);
  return launched();
}

size_t lmce_embedding_grad_workspace_bytes(int64_t n_tokens, int64_t vocab_local) {
  if (n_tokens <= 0 || vocab_local <= 0) return 0;
  return align_up(sizeof(int) * (4 * static_cast<size_t>(vocab_local) + 1), 256) +
         align_up(sizeof(int) * static_cast<size_t>(n_tokens), 256);
}

int lmce_embedding_grad_add(const void* d_embed, const int64_t* token_ids, int64_t n_tokens, int64_t hidden_dim,
                            int64_t vocab_local, int64_t vocab_offset, int dtype, void* d_weight, void* workspace,
                            size_t workspace_bytes, void* stream) {
  if (!d_embed || !token_ids || !d_weight || !workspace) return fail(LMCE_ERR_INVALID_ARGUMENT, "null pointer");
  if (n_tokens <= 0 || n_tokens > (1ll << 30) || vocab_local <= 0 || vocab_local > (1ll << 30) || vocab_offset < 0)
    return fail(LMCE_ERR_INVALID_ARGUMENT, "bad sizes");
  if (hidden_dim <= 0 || hidden_dim % 8 != 0) return fail(LMCE_ERR_INVALID_ARGUMENT, "hidden_dim must be a multiple of 8");
  if (dtype != LMCE_DTYPE_F16 && dtype != LMCE_DTYPE_BF16) return fail(LMCE_ERR_UNSUPPORTED, "dtype %d", dtype);
  if (!aligned16(d_embed) || !aligned16(d_weight) || !aligned16(workspace))
    return fail(LMCE_ERR_INVALID_ARGUMENT, "misaligned buffers");
  if (workspace_bytes < lmce_embedding_grad_workspace_bytes(n_tokens, vocab_local))
    return fail(LMCE_ERR_WORKSPACE, "workspace %zu bytes < required %zu", workspace_bytes,
                lmce_embedding_grad_workspace_bytes(n_tokens, vocab_local));
  DevInfo* d = nullptr;
  if (int rc = device_info(&d)) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int vl = static_cast<int>(vocab_local), h = static_cast<int>(hidden_dim);
  int* counts = static_cast<int*>(workspace);
  int* offsets = counts + vl;
  int* cursor = offsets + vl;
  int* used = cursor + vl;
  int* n_used = used + vl;
  int* order = reinterpret_cast<int*>(static_cast<char*>(workspace) +
                                      align_up(sizeof(int) * (4 * static_cast<size_t>(vl) + 1), 256));
  LMCE_CUDA(cudaMemsetAsync(counts, 0, sizeof(int) * vl, st));
  long long blocks = (n_tokens + 255) / 256;
  if (blocks > d->sms * 4ll) blocks = d->sms * 4ll;
  emb_hist_kernel<<<static_cast<int>(blocks), 256, 0, st>>>(token_ids, n_tokens, vocab_offset, vl, counts);
  if (int rc = launched()) return rc;
  emb_scan_kernel<<<1, PACK_THREADS, 0, st>>>(counts, vl, offsets, cursor, used, n_used);
  if (int rc = launched()) return rc;
  emb_scatter_kernel<<<static_cast<int>(blocks), 256, 0, st>>>(token_ids, n_tokens, vocab_offset, vl, cursor, order);
  if (int rc = launched()) return rc;
  const long long max_used = n_tokens < vocab_local ? n_tokens : vocab_local;  // ids that can occur
  const long long tasks = max_used * ((h + EMB_COLS - 1) / EMB_COLS);
  const long long ablocks = (tasks * 32 + 255) / 256;
  if (ablocks > (1ll << 31) - 1) return fail(LMCE_ERR_UNSUPPORTED, "too many rows");
  if (dtype == LMCE_DTYPE_BF16)
    emb_accumulate_kernel<true><<<static_cast<int>(ablocks), 256, 0, st>>>(
        static_cast<const uint4*>(d_embed), h, used, n_used, counts, offsets, order, static_cast<uint4*>(d_weight));
  else
    emb_accumulate_kernel<false><<<static_cast<int>(ablocks), 256, 0, st>>>(
        static_cast<const uint4*>(d_embed), h, used, n_used, counts, offsets, order, static_cast<uint4*>(d_weight));
  return launched();
}

int lmce_embedding_lookup(const void* weight, const int64_t* token_ids, int64_t n_tokens, int64_t hidden_dim,
                          int64_t vocab_local, int64_t vocab_offset, void* out, void* stream) {
  if (!weight || !token_ids || !out) return fail(LMCE_ERR_INVALID_ARGUMENT, "null pointer");
  if (n_tokens <= 0 || vocab_local <= 0 || vocab_offset < 0) return fail(LMCE_ERR_INVALID_ARGUMENT, "bad sizes");
  if (hidden_dim <= 0 || hidden_dim % 8 != 0) return fail(LMCE_ERR_INVALID_ARGUMENT, "hidden_dim must be a multiple of 8");
  if (!aligned16(weight) || !aligned16(out)) return fail(LMCE_ERR_INVALID_ARGUMENT, "misaligned buffers");
  DevInfo* d = nullptr;
  if (int rc = device_info(&d)) return rc;
  const int vec = static_cast<int>(hidden_dim * 2 / 16);
  long long blocks = (n_tokens * vec + 255) / 256;
  if (blocks > d->sms * 8ll) blocks = d->sms * 8ll;
  emb_lookup_kernel<<<static_cast<int>(blocks), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint4*>(weight), token_ids, n_tokens, vec, vocab_offset, static_cast<int>(vocab_local),
      static_cast<uint4*>(out));
  return launched();
}

int lmce_rmsnorm_pack(const void* hidden, const void* weight, float eps, const int64_t* row_idx,
                      const int32_t* count, int64_t n_rows, int64_t hidden_dim, int dtype, void* x_out,
                      float* rstd_out, void* stream) {
  if (!hidden || !weight || !x_out || !rstd_out) return fail(LMCE_ERR_INVALID_ARGUMENT, "null pointer");
  if (n_rows <= 0 || n_rows > (1ll << 30)) return fail(LMCE_ERR_INVALID_ARGUMENT, "bad n_rows");
  if (hidden_dim <= 0 || hidden_dim % 8 != 0) return fail(LMCE_ERR_INVALID_ARGUMENT, "hidden_dim must be a multiple of 8");
  if (dtype != LMCE_DTYPE_F16 && dtype != LMCE_DTYPE_BF16) return fail(LMCE_ERR_UNSUPPORTED, "dtype %d", dtype);
  if (!aligned16(hidden) || !aligned16(weight) || !aligned16(x_out)) return fail(LMCE_ERR_INVALID_ARGUMENT, "misaligned buffers");
  DevInfo* d = nullptr;
  if (int rc = device_info(&d)) return rc;
  const int vec = static_cast<int>(hidden_dim / 8);
  long long blocks = (n_rows * 32 + 255) / 256;
  if (blocks > d->sms * 16ll) blocks = d->sms * 16ll;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const float inv = 1.0f / static_cast<float>(hidden_dim);
  if (dtype == LMCE_DTYPE_BF16)
    rmsnorm_pack_kernel<true><<<static_cast<int>(blocks), 256, 0, st>>>(
        static_cast<const uint4*>(hidden), static_cast<const uint4*>(weight), row_idx, count, n_rows, vec, inv, eps,
        static_cast<uint4*>(x_out), rstd_out);
  else
    rmsnorm_pack_kernel<false><<<static_cast<int>(blocks), 256, 0, st>>>(
        static_cast<const uint4*>(hidden), static_cast<const uint4*>(weight), row_idx, count, n_rows, vec, inv, eps,
        static_cast<uint4*>(x_out), rstd_out);
  return launched();
}

int lmce_rmsnorm_backward(const void* d_x, const void* hidden, const void* weight, const float* rstd,
                          const int64_t* row_idx, const int32_t* count, int64_t n_rows, int64_t hidden_dim, int dtype,
                          void* d_hidden, void* stream) {
  if (!d_x || !hidden || !weight || !rstd || !d_hidden) return fail(LMCE_ERR_INVALID_ARGUMENT, "null pointer");
  if (n_rows <= 0 || n_rows > (1ll << 30)) return fail(LMCE_ERR_INVALID_ARGUMENT, "bad n_rows");
  if (hidden_dim <= 0 || hidden_dim % 8 != 0) return fail(LMCE_ERR_INVALID_ARGUMENT, "hidden_dim must be a multiple of 8");
  if (dtype != LMCE_DTYPE_F16 && dtype != LMCE_DTYPE_BF16) return fail(LMCE_ERR_UNSUPPORTED, "dtype %d", dtype);
  if (!aligned16(d_x) || !aligned16(hidden) || !aligned16(weight) || !aligned16(d_hidden))
    return fail(LMCE_ERR_INVALID_ARGUMENT, "misaligned buffers");
  DevInfo* d = nullptr;
  if (int rc = device_info(&d)) return rc;
  const int vec = static_cast<int>(hidden_dim / 8);
  long long blocks = (n_rows * 32 + 255) / 256;
  if (blocks > d->sms * 16ll) blocks = d->sms * 16ll;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const float inv = 1.0f / static_cast<float>(hidden_dim);
  if (dtype == LMCE_DTYPE_BF16)
    rmsnorm_backward_kernel<true><<<static_cast<int>(blocks), 256, 0, st>>>(
        static_cast<const uint4*>(d_x), static_cast<const uint4*>(hidden), static_cast<const uint4*>(weight), rstd,
        row_idx, count, n_rows, vec, inv, static_cast<uint4*>(d_hidden));
  else
    rmsnorm_backward_kernel<false><<<static_cast<int>(blocks), 256, 0, st>>>(
        static_cast<const uint4*>(d_x), static_cast<const uint4*>(hidden), static_cast<const uint4*>(weight), rstd,
        row_idx, count, n_rows, vec, inv, static_cast<uint4*>(d_hidden));
  return launched();
}

int lmce_selftest_wait_timeout(uint64_t timeout_ns, void* stream) {
  DevInfo* d = nullptr;
  if (int rc = device_info(&d)) return rc;
  selftest_wait_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(timeout_ns, d->err_ptr);
  return launched();
}

uint64_t lmce_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

int lmce_probe_tma_pipeline(const void* tensor, int64_t rows, int64_t cols, int load_kind, int stage_bytes,
                            int stages, int hold_cycles, int iters, unsigned long long* cycles, int64_t n_cycles,
                            void* stream) {
  if (!tensor || !cycles) return fail(LMCE_ERR_INVALID_ARGUMENT, "null pointer");
  if (reinterpret_cast<uintptr_t>(tensor) % 16 != 0) return fail(LMCE_ERR_INVALID_ARGUMENT, "tensor not 16-byte aligned");
  if (rows < 128 || rows % 128 != 0 || cols < 128 || cols % 128 != 0)
    return fail(LMCE_ERR_INVALID_ARGUMENT, "rows and cols must be positive multiples of 128");
  if (load_kind < 0 || load_kind > 2) return fail(LMCE_ERR_INVALID_ARGUMENT, "load_kind must be 0, 1 or 2");
  const int piece = load_kind == 0 ? 16384 : 32768;
  if (stage_bytes < piece || stage_bytes % piece != 0)
    return fail(LMCE_ERR_INVALID_ARGUMENT, "stage_bytes must be a positive multiple of %d for load_kind %d", piece,
                load_kind);
  if (stages < 2 || stages > PROBE_MAX_STAGES) return fail(LMCE_ERR_INVALID_ARGUMENT, "stages must be 2..8");
  const long long smem = static_cast<long long>(stages) * stage_bytes + 2048;
  if (smem > PROBE_MAX_SMEM) return fail(LMCE_ERR_INVALID_ARGUMENT, "stages x stage_bytes exceeds shared memory");
  if (hold_cycles < 0 || hold_cycles > 1000000) return fail(LMCE_ERR_INVALID_ARGUMENT, "hold_cycles out of range");
  if (iters < 16) return fail(LMCE_ERR_INVALID_ARGUMENT, "iters must be at least 16");
  DevInfo* d = nullptr;
  if (int rc = device_info(&d)) return rc;
  if (n_cycles < d->sms) return fail(LMCE_ERR_INVALID_ARGUMENT, "cycles needs one entry per SM (%d)", d->sms);
  if (int rc = get_encoder()) return rc;
  CUtensorMap m2, m3;
  if (int rc = make_map(&m2, tensor, false, cols, rows, cols, 128)) return rc;
  if (int rc = make_map_3d(&m3, tensor, false, cols, rows, cols, 128, 2)) return rc;
  auto kern = tma_pipeline_probe_kernel;
  static bool done[kMaxDevices] = {};
  if (int rc = ensure_smem_attr(kern, PROBE_MAX_SMEM, done)) return rc;
  const long long n_pieces32 = rows * cols * 2 / 32768;
  kern<<<d->sms, 64, static_cast<size_t>(smem), static_cast<cudaStream_t>(stream)>>>(
      m2, m3, static_cast<const uint8_t*>(tensor), n_pieces32, load_kind, stage_bytes, stages, hold_cycles, iters,
      static_cast<int>(rows / 128), static_cast<int>(cols / 64), wait_timeout_ns(), cycles, d->err_ptr);
  return launched();
}

int lmce_probe_tma_rate(const void* tensor, int64_t rows, int64_t cols, int box_kind, int iters,
                        unsigned long long* cycles, int64_t n_cycles, void* stream) {
  if (box_kind != 0 && box_kind != 1) return fail(LMCE_ERR_INVALID_ARGUMENT, "box_kind must be 0 or 1");
  return lmce_probe_tma_pipeline(tensor, rows, cols, box_kind, 32768, 3, 0, iters, cycles, n_cycles, stream);
}

int lmce_profile_read(void* counters, size_t counter_bytes, void* timeline, size_t timeline_bytes, int reset) {
#if LMCE_ROLE_PROFILE
  if (counter_bytes > sizeof(g_prof_ctr) || timeline_bytes > sizeof(g_prof_tl))
    return fail(LMCE_ERR_INVALID_ARGUMENT, "profile buffers larger than the device arrays");
  if (counters && counter_bytes) LMCE_CUDA(cudaMemcpyFromSymbol(counters, g_prof_ctr, counter_bytes));
  if (timeline && timeline_bytes) LMCE_CUDA(cudaMemcpyFromSymbol(timeline, g_prof_tl, timeline_bytes));
  if (reset) {
    void* p = nullptr;
    LMCE_CUDA(cudaGetSymbolAddress(&p, g_prof_ctr));
    LMCE_CUDA(cudaMemset(p, 0, sizeof(g_prof_ctr)));
    LMCE_CUDA(cudaGetSymbolAddress(&p, g_prof_tl));
    LMCE_CUDA(cudaMemset(p, 0, sizeof(g_prof_tl)));
  }
  return LMCE_OK;
#else
  (void)counters;
  (void)counter_bytes;
  (void)timeline;
  (void)timeline_bytes;
  (void)reset;
  return fail(LMCE_ERR_UNSUPPORTED, "built without LMCE_ROLE_PROFILE");
#endif
}

int lmce_set_timing_events(int which, void* begin, void* end) {
  if (which < 0 || which > 1) return fail(LMCE_ERR_INVALID_ARGUMENT, "timing slot %d", which);
  if ((begin == nullptr) != (end == nullptr)) return fail(LMCE_ERR_INVALID_ARGUMENT, "set both events or neither");
  if (begin != nullptr && g_event_record == nullptr) {
    static std::once_flag once;
    std::call_once(once, [] {
      cudaDriverEntryPointQueryResult q;
      void* fn = nullptr;
      if (cudaGetDriverEntryPoint("cuEventRecord", &fn, cudaEnableDefault, &q) == cudaSuccess &&
          q == cudaDriverEntryPointSuccess)
        g_event_record = reinterpret_cast<PFN_cuEventRecord_v2000>(fn);
    });
    if (g_event_record == nullptr) return fail(LMCE_ERR_CUDA, "cuEventRecord unavailable");
  }
  g_timing[which][0].store(static_cast<CUevent>(begin), std::memory_order_release);
  g_timing[which][1].store(static_cast<CUevent>(end), std::memory_order_release);
  return LMCE_OK;
}

}  // extern "C"

// ======================================================= no-allocation forward ===
//
// Scratch for lmce_forward_noalloc: a fixed device array inside this library, so
// a caller that cannot allocate device memory can still run the forward. Host
// code never passes the symbol itself to a kernel (on the host it names a
// stand-in, not device memory); it looks up the device address once per device
// with cudaGetSymbolAddress and passes that pointer.

static __device__ __align__(256) unsigned char g_lmce_noalloc_scratch[LMCE_NOALLOC_SCRATCH_BYTES];

namespace {

void* g_noalloc_ptr[kMaxDevices] = {};
std::mutex g_noalloc_mu;

// Device address of the scratch array on the current device (looked up on the first call per device).
int noalloc_scratch(void** out) {
  int dev = 0;
  LMCE_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) return fail(LMCE_ERR_UNSUPPORTED, "device ordinal %d out of range", dev);
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (g_noalloc_ptr[dev] == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_lmce_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr)
      return fail(LMCE_ERR_CUDA, "cudaGetSymbolAddress(no-allocation scratch) failed: %s", cudaGetErrorString(e));
    g_noalloc_ptr[dev] = p;
  }
  *out = g_noalloc_ptr[dev];
  return LMCE_OK;
}

}  // namespace

extern "C" int lmce_forward_noalloc(const void* hidden, const void* weight, const int64_t* labels, int64_t n_tokens,
                                    int64_t hidden_dim, int64_t vocab, int dtype, const float* num_items_dev,
                                    double num_items, float* lse, float* nll, float* entropy, int64_t* argmax,
                                    float* loss, float* denom, void* stream) {
  constexpr int64_t kMaxRecords = static_cast<int64_t>(LMCE_NOALLOC_SCRATCH_BYTES / sizeof(lmce_part));
  // every argument is checked before anything is queued, so a rejected call leaves the
  // shared scratch (the previous call's records) untouched
  if (!hidden || !weight || !labels || !lse || !nll || !entropy || !argmax || !loss || !denom)
    return fail(LMCE_ERR_INVALID_ARGUMENT, "null pointer");
  if (!aligned16(hidden) || !aligned16(weight)) return fail(LMCE_ERR_INVALID_ARGUMENT, "hidden/weight not 16-byte aligned");
  if (dtype != LMCE_DTYPE_F16 && dtype != LMCE_DTYPE_BF16) return fail(LMCE_ERR_UNSUPPORTED, "dtype %d", dtype);
  if (hidden_dim <= 0 || hidden_dim % 64 != 0) return fail(LMCE_ERR_UNSUPPORTED, "hidden_dim must be a positive multiple of 64");
  if (n_tokens <= 0) return fail(LMCE_ERR_INVALID_ARGUMENT, "bad n_tokens %lld", (long long)n_tokens);
  if (n_tokens > kMaxRecords)
    return fail(LMCE_ERR_INVALID_ARGUMENT,
                "n_tokens %lld exceeds the no-allocation scratch: %u bytes hold at most %lld tokens "
                "(use lmce_fwd_stats with a caller-allocated buffer)",
                (long long)n_tokens, LMCE_NOALLOC_SCRATCH_BYTES, (long long)kMaxRecords);
  if (vocab <= 0) return fail(LMCE_ERR_INVALID_ARGUMENT, "bad vocab size");
  // vocab slabs per token block, capped so n_tokens x slabs records fit the scratch
  int64_t parts = lmce_fwd_num_parts(n_tokens, vocab);
  const int64_t cap = kMaxRecords / n_tokens;
  if (parts > cap) parts = cap;
  if (parts < 1) parts = 1;
  void* scratch = nullptr;
  if (int rc = noalloc_scratch(&scratch)) return rc;
  lmce_part* recs = static_cast<lmce_part*>(scratch);
  if (int rc = lmce_fwd_stats(hidden, weight, labels, n_tokens, hidden_dim, vocab, 0, dtype, recs, parts, stream))
    return rc;
  return lmce_stats_finish(recs, parts, parts, 1, labels, n_tokens, num_items_dev, num_items, lse, nll, entropy,
                           argmax, loss, denom, stream);
}
