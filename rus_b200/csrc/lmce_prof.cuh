// Role counters of the persistent backward, compiled in only with -DLMCE_ROLE_PROFILE=1.
//
// The product build defines nothing here beyond empty macros. A profiling build
// keeps, per CTA, PROF_SLOTS cycle counters (clock64) of where each role of the
// kernel spent its time, and per tile one timeline entry (globaltimer ns) written
// by the first epilogue thread (the UMMA issuer adds its start time to the same
// entry: both consume the schedule ring in the same order). lmce_profile_read()
// copies them out; lmce_profile_reset() clears them.
#pragma once

#ifndef LMCE_ROLE_PROFILE
#define LMCE_ROLE_PROFILE 0
#endif

#if LMCE_ROLE_PROFILE
#define LMCE_PROF(...) __VA_ARGS__
#else
#define LMCE_PROF(...)
#endif

namespace lmce {

// Counter slots (one block of PROF_SLOTS per CTA).
enum : int {
  PS_TOTAL = 0,        // kernel body cycles (thread 0, after set-up to the final barrier)
  PS_P_SCHED = 1,      // producer: schedule ring waits (leader: free slot; peer: next tile)
  PS_P_DEP_G = 2,      // producer: G-buffer release waits before a GT tile
  PS_P_DEP_GD = 3,     // producer: G-complete waits before DX / DW tiles
  PS_P_EMPTY = 4,      // producer: free-stage waits
  PS_P_TILES = 5,      // producer: tiles loaded
  PS_M_SCHED = 6,      // UMMA issuer: waits for the next tile
  PS_M_TEMPTY = 7,     // UMMA issuer: waits for a free accumulator
  PS_M_FULL_G = 8,     // UMMA issuer: full-stage waits, by tile kind
  PS_M_FULL_DX = 9,
  PS_M_FULL_DW = 10,
  PS_M_KB_G = 11,      // UMMA issuer: k-blocks issued, by tile kind
  PS_M_KB_DX = 12,
  PS_M_KB_DW = 13,
  PS_M_LOOP = 15,      // UMMA issuer: whole loop
  PS_E_SCHED = 16,     // first epilogue thread: waits for the next tile
  PS_E_CHAIN = 17,     // waits on the dX chain (DX(c-1) of the same tile)
  PS_E_TFULL_G = 18,   // waits for the accumulator, by tile kind
  PS_E_TFULL_DX = 19,
  PS_E_TFULL_DW = 20,
  PS_E_WORK_G = 21,    // accumulator ready -> tile published, by tile kind
  PS_E_WORK_DX = 22,
  PS_E_WORK_DW = 23,
  PS_E_XCH = 24,       // exchange items
  PS_E_N_G = 25,       // tiles, by kind
  PS_E_N_DX = 26,
  PS_E_N_DW = 27,
  PS_E_LOOP = 28,      // whole epilogue loop
  PROF_SLOTS = 32
};

constexpr int PROF_MAX_CTAS = 256;
constexpr int PROF_TILES = 1024;  // timeline entries per CTA
constexpr int PROF_ENTRY = 8;     // u64 per entry: kind, chunk, m, n, t_mma_start, t_sched, t_tfull, t_done

#if LMCE_ROLE_PROFILE
__device__ unsigned long long g_prof_ctr[PROF_MAX_CTAS * PROF_SLOTS];
__device__ unsigned long long g_prof_tl[PROF_MAX_CTAS * PROF_TILES * PROF_ENTRY];

__device__ __forceinline__ void prof_store(int slot, unsigned long long v) {
  if (blockIdx.x < PROF_MAX_CTAS) g_prof_ctr[blockIdx.x * PROF_SLOTS + slot] = v;
}

__device__ __forceinline__ unsigned long long* prof_entry(int i) {
  return (blockIdx.x < PROF_MAX_CTAS && i < PROF_TILES)
             ? &g_prof_tl[(static_cast<size_t>(blockIdx.x) * PROF_TILES + i) * PROF_ENTRY]
             : nullptr;
}
#endif

}  // namespace lmce
