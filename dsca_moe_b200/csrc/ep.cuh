// Expert-parallel device context shared by the plan / dispatch / wait kernels (ep.cu) and the
// grouped GEMM's return epilogue (gemm_sm100.cu).
//
// Every rank owns one symmetric region (same layout on every rank, mapped into every peer
// through CUDA IPC): flags [4][kMaxG] u32 (counts / dispatch / return / priorities, written by
// the source rank with release semantics, value = the forward's epoch), meta [kMaxG][kMaxE] i32 (each
// source's per-expert counts), the receive buffer (rows dispatched to this rank, expert-major)
// and the return buffer (this rank's expert outputs coming back, in its send layout).
#pragma once

#include "common.cuh"

namespace dsca {
namespace ep {

constexpr int kMaxG = DSCA_MAX_GPUS;      // 8
constexpr int kCtasPerSm = 2;             // resident CTAs per SM of the dispatch / return copy kernels
constexpr int kMaxE = DSCA_MAX_EXPERTS;   // 64
enum FlagKind { kCounts = 0, kDispatch = 1, kReturn = 2, kPrio = 3 };

struct Ctx {
  int G, E, me, d;
  int recv_capacity, ret_capacity, eq_tokens, elem_bytes;
  uint32_t epoch;          // epoch of the forward in flight (the plan kernel advances it)
  uint32_t dispatch_done;  // CTA completion counters (last CTA signals the peers, then resets)
  uint32_t return_done;
  int32_t recv_total;
  int32_t expert_to_gpu[kMaxE];
  uint32_t* flags[kMaxG];  // flags[p]: peer p's flag array [3][kMaxG]
  int32_t* meta[kMaxG];    // meta[p]:  peer p's counts table [kMaxG][kMaxE], then its priority
                           //           table [kMaxG][kMaxE] (fp32 bits) right after it
  char* recv[kMaxG];       // recv[p]:  peer p's receive buffer
  char* ret[kMaxG];        // ret[p]:   peer p's return buffer
  // plan tables (written on the device by the plan kernel each forward)
  int32_t group_offsets[kMaxE + 1];        // this rank's receive buffer, expert-major
  int32_t cum_split[kMaxE][kMaxG];         // inclusive prefix over dst of S[me][e][dst]
  int32_t remote_base[kMaxE][kMaxG];       // first row of chunk (me, e) in dst's receive buffer
  int32_t send_base[kMaxE][kMaxG];         // first row of (e, dst) in this rank's send layout
  int32_t chunk_start[kMaxE][kMaxG];       // first row of chunk (src, e) in this receive buffer
  int32_t chunk_len[kMaxE][kMaxG];         // S[src][e][me]
  int32_t ret_start[kMaxE][kMaxG];         // where chunk (src, e) goes in src's return buffer
  int32_t S[kMaxG][kMaxE][kMaxG];          // the plan
  // QoS execution order: experts by the priority summed over the ranks (descending, lowest id on
  // ties); position -> expert.  The identity when the forward carries no priorities.
  int32_t group_order[kMaxE];
  float priority[kMaxE];                   // the summed priorities of the last forward
  uint32_t prio_epoch;  // epoch of the last priority exchange (dsca_ep_priority advances it)
};

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Bounded wait until *p == v (epochs only grow, so >= is used).  Returns false after the limit.
__device__ __forceinline__ bool wait_flag(const uint32_t* p, uint32_t v, uint64_t limit_ns) {
  if ((int32_t)(ld_acquire_sys(p) - v) >= 0) return true;
  const uint64_t t0 = globaltimer_ns();
  while (true) {
    __nanosleep(64);
    if ((int32_t)(ld_acquire_sys(p) - v) >= 0) return true;
    if (globaltimer_ns() - t0 > limit_ns) return false;
  }
}

// Copy one row of nvec 16-byte vectors with a warp (lane-strided, so each store instruction
// covers 512 contiguous bytes), eight loads in flight per lane before the stores go out.
__device__ __forceinline__ void warp_copy_row(uint4* __restrict__ dst, const uint4* __restrict__ src, int nvec,
                                              int lane) {
  int v = lane;
  for (; v + 7 * 32 < nvec; v += 8 * 32) {
    uint4 r[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) r[i] = src[v + 32 * i];
#pragma unroll
    for (int i = 0; i < 8; ++i) dst[v + 32 * i] = r[i];
  }
  for (; v < nvec; v += 32) dst[v] = src[v];
}

// Last-CTA-done signal: every thread fences its own stores (system scope), the CTA counts
// itself in; the last CTA tells every peer (flag kind `kind`, value = epoch) and resets the
// counter for the next forward.  Called by every thread of the CTA.
__device__ __forceinline__ void signal_when_grid_done(Ctx* c, uint32_t* counter, int kind) {
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    const uint32_t prev = atomicAdd(counter, 1u);
    if (prev == gridDim.x - 1) {
      *counter = 0u;
      __threadfence_system();
      const uint32_t epoch = *reinterpret_cast<volatile uint32_t*>(&c->epoch);
      for (int p = 0; p < c->G; ++p) st_release_sys(c->flags[p] + kind * kMaxG + c->me, epoch);
    }
  }
}

}  // namespace ep
}  // namespace dsca
