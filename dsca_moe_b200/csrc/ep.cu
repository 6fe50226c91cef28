// Fused expert-parallel exchange over NVLink peer memory (one process per GPU, CUDA IPC).
//
//   plan kernel     counts of this rank -> every peer's meta table (P2P stores), epoch flag,
//                   bounded wait for every peer's counts, then the harmony plan and the send /
//                   receive tables computed on the device by one warp (the same integer algorithm
//                   as dsca_plan_harmony, src/harmonymoe/scheduler.py:324-372, and
//                   dsca_plan_layout, :101-124 / :185-213) — no host sync anywhere.
//   dispatch kernel every routed (token, slot) row stored straight into the destination rank's
//                   expert-major receive buffer (16-byte stores over NVLink); the last CTA sets
//                   the dispatch flag at every peer.
//   wait kernel     bounded wait for one flag kind from every peer.
// The grouped GEMM's return epilogue (gemm_sm100.cu) stores expert outputs straight into the
// source rank's return buffer and sets the return flag.  Peer memory is only ever the target of
// plain stores or the source of plain loads: no TMA and no multicast touches it.
#include <string.h>

#include <algorithm>

#include "ep.cuh"

namespace dsca {
namespace ep {

// ------------------------------------------------------------------ harmony plan, one warp
// S (shared) [G][E][G]; meta [G][E]; all lanes call it, control flow is warp-uniform.
// Reference form with 64-bit sums and shuffle reductions (used when the token total does not fit
// the packed keys of harmony_warp_fast below).
__device__ void harmony_warp_wide(const int32_t* meta, int G, int E, const int32_t* e2g, int eq_tokens, int32_t* S,
                                  long long* amt) {
  const int lane = threadIdx.x & 31;
  for (int i = lane; i < G * E * G; i += 32) S[i] = 0;
  __syncwarp();
  long long part = 0;
  for (int i = lane; i < G * E; i += 32) {
    const int src = i / E, e = i % E;
    S[(src * E + e) * G + e2g[e]] = meta[i];
    part += meta[i];
  }
  for (int off = 16; off; off >>= 1) part += __shfl_xor_sync(0xffffffffu, part, off);
  const long long total = part;
  __syncwarp();
  if (eq_tokens < 0) return;
  const long long avg = total / G;
  if (lane < G) {
    long long a = 0;
    for (int src = 0; src < G; ++src)
      for (int e = 0; e < E; ++e) a += S[(src * E + e) * G + lane];
    amt[lane] = a;
  }
  __syncwarp();
  for (int guard = 0; guard < (1 << 20); ++guard) {
    // most / least loaded GPU (first index on ties)
    long long mv = lane < G ? amt[lane] : LLONG_MIN, lv = lane < G ? amt[lane] : LLONG_MAX;
    int mi = lane < G ? lane : 1 << 30, li = mi;
    bool over_any = lane < G && amt[lane] > avg;
    over_any = __any_sync(0xffffffffu, over_any);
    if (!over_any) break;
    for (int off = 16; off; off >>= 1) {
      long long ov = __shfl_xor_sync(0xffffffffu, mv, off);
      int oi = __shfl_xor_sync(0xffffffffu, mi, off);
      if (ov > mv || (ov == mv && oi < mi)) { mv = ov; mi = oi; }
      long long lv2 = __shfl_xor_sync(0xffffffffu, lv, off);
      int li2 = __shfl_xor_sync(0xffffffffu, li, off);
      if (lv2 < lv || (lv2 == lv && li2 < li)) { lv = lv2; li = li2; }
    }
    const int over = mi, least = li;
    if (least == over || amt[least] + eq_tokens > avg) break;
    // the expert with most tokens on the overloaded GPU
    long long sv = LLONG_MIN;
    int si = 1 << 30;
    for (int e = lane; e < E; e += 32) {
      long long s = 0;
      for (int src = 0; src < G; ++src) s += S[(src * E + e) * G + over];
      if (s > sv) { sv = s; si = e; }
    }
    for (int off = 16; off; off >>= 1) {
      long long ov = __shfl_xor_sync(0xffffffffu, sv, off);
      int oi = __shfl_xor_sync(0xffffffffu, si, off);
      if (ov > sv || (ov == sv && oi < si)) { sv = ov; si = oi; }
    }
    const int e = si;
    if (sv < eq_tokens) break;
    long long amount_over = amt[over] - avg;
    long long moved = 0;
    while (amount_over > 0 && avg - amt[least] > 0) {
      long long tv = lane < G ? (long long)S[(lane * E + e) * G + over] : LLONG_MIN;
      int ti = lane < G ? lane : 1 << 30;
      for (int off = 16; off; off >>= 1) {
        long long ov = __shfl_xor_sync(0xffffffffu, tv, off);
        int oi = __shfl_xor_sync(0xffffffffu, ti, off);
        if (ov > tv || (ov == tv && oi < ti)) { tv = ov; ti = oi; }
      }
      if (tv <= 0) break;
      const long long room = avg - amt[least];
      const long long n = tv < room ? tv : room;
      __syncwarp();
      if (lane == 0) {
        S[(ti * E + e) * G + over] -= (int32_t)n;
        S[(ti * E + e) * G + least] += (int32_t)n;
        amt[over] -= n;
        amt[least] += n;
      }
      __syncwarp();
      amount_over -= n;
      moved += n;
    }
    if (moved == 0) break;
  }
  __syncwarp();
}

// The same plan with every arg-max / arg-min as one warp reduction over a packed (value, index)
// key (value << bits | index or its complement, so ties go to the lowest index exactly as in the
// reference's first-index scans) and the per-expert load of each GPU kept in Le[e][g] instead
// of being re-summed over the sources on every pass.  Token totals below 2^26.
__device__ void harmony_warp(const int32_t* meta, int G, int E, const int32_t* e2g, int eq_tokens, int32_t* S,
                             long long* amt_wide, int32_t* Le, int32_t* amt) {
  const int lane = threadIdx.x & 31;
  const unsigned full = 0xffffffffu;
  int part = 0;
  for (int i = lane; i < G * E; i += 32) part += meta[i];
  const unsigned total = __reduce_add_sync(full, (unsigned)part);
  if (total >= (1u << 26)) {
    harmony_warp_wide(meta, G, E, e2g, eq_tokens, S, amt_wide);
    return;
  }
  for (int i = lane; i < G * E * G; i += 32) S[i] = 0;
  for (int i = lane; i < E * G; i += 32) Le[i] = 0;
  __syncwarp();
  for (int i = lane; i < G * E; i += 32) {
    const int src = i / E, e = i % E;
    S[(src * E + e) * G + e2g[e]] = meta[i];
  }
  for (int e = lane; e < E; e += 32) {
    int se = 0;
    for (int src = 0; src < G; ++src) se += meta[src * E + e];
    Le[e * G + e2g[e]] = se;
  }
  __syncwarp();
  if (eq_tokens < 0) return;
  const int avg = (int)(total / (unsigned)G);
  if (lane < G) {
    int a = 0;
    for (int e = 0; e < E; ++e) a += Le[e * G + lane];
    amt[lane] = a;
  }
  __syncwarp();
  for (int guard = 0; guard < (1 << 20); ++guard) {
    const int a = lane < G ? amt[lane] : 0;
    if (!__any_sync(full, lane < G && a > avg)) break;
    // most loaded GPU (lowest index on ties) and least loaded GPU (lowest index on ties)
    const unsigned mk = __reduce_max_sync(full, lane < G ? ((unsigned)a << 5) | (31u - lane) : 0u);
    const unsigned lk = __reduce_min_sync(full, lane < G ? ((unsigned)a << 5) | (unsigned)lane : 0xffffffffu);
    const int over = 31 - (int)(mk & 31u), least = (int)(lk & 31u);
    if (least == over || amt[least] + eq_tokens > avg) break;
    // the expert with most tokens on the overloaded GPU (lowest id on ties)
    unsigned ek = 0u;
    for (int e = lane; e < E; e += 32) ek = max(ek, ((unsigned)Le[e * G + over] << 6) | (63u - e));
    ek = __reduce_max_sync(full, ek);
    const int e = 63 - (int)(ek & 63u);
    if ((int)(ek >> 6) < eq_tokens) break;
    int amount_over = amt[over] - avg;
    int moved = 0;
    while (amount_over > 0 && avg - amt[least] > 0) {
      // the source rank with most tokens of expert e on `over` (lowest rank on ties)
      const unsigned tk = __reduce_max_sync(
          full, lane < G ? ((unsigned)S[(lane * E + e) * G + over] << 5) | (31u - lane) : 0u);
      const int tv = (int)(tk >> 5), ti = 31 - (int)(tk & 31u);
      if (tv <= 0) break;
      const int room = avg - amt[least];
      const int n = tv < room ? tv : room;
      __syncwarp();
      if (lane == 0) {
        S[(ti * E + e) * G + over] -= n;
        S[(ti * E + e) * G + least] += n;
        Le[e * G + over] -= n;
        Le[e * G + least] += n;
        amt[over] -= n;
        amt[least] += n;
      }
      __syncwarp();
      amount_over -= n;
      moved += n;
    }
    if (moved == 0) break;
  }
  __syncwarp();
}

// QoS execution order from the priority tables every rank pushed into meta[me] (summed over
// the ranks in rank order: the all-reduce of src/qosmoe/moe_layer.py:379-380, identical on
// every rank), descending, lowest expert id on ties (the stable sort of build_exec_plan,
// src/qosmoe/planner.py:189-198, with every expert resident).  Threads < E; ends with a
// __syncthreads.
__device__ __forceinline__ void qos_order(Ctx* c, bool have_priority, float* prio_s) {
  const int E = c->E, G = c->G, tid = threadIdx.x;
  const volatile int32_t* ml = c->meta[c->me];
  if (tid < E) {
    float sum = 0.0f;
    if (have_priority)
      for (int src = 0; src < G; ++src) sum = __fadd_rn(sum, __int_as_float(ml[kMaxG * kMaxE + src * kMaxE + tid]));
    prio_s[tid] = (sum == sum) ? sum : -INFINITY;  // a NaN orders last: the order stays a permutation
  }
  __syncthreads();
  if (tid < E) {
    const float pe = prio_s[tid];
    int pos = 0;
    for (int e2 = 0; e2 < E; ++e2) {
      const float q = prio_s[e2];
      pos += (q > pe || (q == pe && e2 < tid)) ? 1 : 0;
    }
    c->group_order[pos] = tid;
    c->priority[tid] = pe;
  }
  __syncthreads();
}

// ------------------------------------------------------------------ priority kernel
// dsca_ep_priority: this rank's [E] priorities into every rank's priority table, the kPrio flag,
// a bounded wait for every rank's, then the execution order.  Its own epoch, so it may run beside
// the counts-only plan of the same forward on another stream.
__global__ void __launch_bounds__(256) priority_kernel(Ctx* c, const float* priority, uint64_t limit_ns,
                                                       int32_t* err) {
  __shared__ float prio_s[kMaxE];
  const int G = c->G, E = c->E, me = c->me, tid = threadIdx.x;
  const uint32_t epoch = *reinterpret_cast<volatile uint32_t*>(&c->prio_epoch) + 1u;
  for (int i = tid; i < G * E; i += blockDim.x) {
    const int p = i / E, e = i % E;
    c->meta[p][kMaxG * kMaxE + me * kMaxE + e] = __float_as_int(priority[e]);
  }
  __syncthreads();
  if (tid == 0) {
    __threadfence_system();
    for (int p = 0; p < G; ++p) st_release_sys(c->flags[p] + kPrio * kMaxG + me, epoch);
  }
  if (tid < G) {
    if (!wait_flag(c->flags[me] + kPrio * kMaxG + tid, epoch, limit_ns)) record_error(err, kErrWaitTimeout);
  }
  __syncthreads();
  qos_order(c, true, prio_s);
  if (tid == 0) {
    __threadfence();
    *reinterpret_cast<volatile uint32_t*>(&c->prio_epoch) = epoch;
  }
}

// ------------------------------------------------------------------ plan kernel
// kOrder = false (dsca_ep_plan_counts): counts only; the QoS order and the priority tables are
// left to dsca_ep_priority.
template <bool kOrder>
__global__ void __launch_bounds__(256) plan_kernel(Ctx* c, const int32_t* counts, const float* priority,
                                                   uint64_t limit_ns, int32_t* err) {
  __shared__ int32_t meta_s[kMaxG * kMaxE];
  __shared__ int32_t S_s[kMaxG * kMaxE * kMaxG];
  __shared__ long long amt_s[kMaxG];
  __shared__ int32_t amt32_s[kMaxG];
  __shared__ int32_t le_s[kMaxE * kMaxG];
  __shared__ int32_t e2g_s[kMaxE];
  const int G = c->G, E = c->E, me = c->me, tid = threadIdx.x;
  const uint32_t epoch = *reinterpret_cast<volatile uint32_t*>(&c->epoch) + 1u;
  // 1. my counts (and QoS priorities) into every rank's meta[me][*]
  for (int i = tid; i < G * E; i += blockDim.x) {
    const int p = i / E, e = i % E;
    c->meta[p][me * kMaxE + e] = counts[e];
    if (kOrder && priority != nullptr) c->meta[p][kMaxG * kMaxE + me * kMaxE + e] = __float_as_int(priority[e]);
  }
  __syncthreads();
  if (tid == 0) {
    __threadfence_system();
    for (int p = 0; p < G; ++p) st_release_sys(c->flags[p] + kCounts * kMaxG + me, epoch);
  }
  // 2. every rank's counts
  if (tid < G) {
    if (!wait_flag(c->flags[me] + kCounts * kMaxG + tid, epoch, limit_ns)) record_error(err, kErrWaitTimeout);
  }
  __syncthreads();
  const volatile int32_t* ml = c->meta[me];
  for (int i = tid; i < G * E; i += blockDim.x) meta_s[i] = ml[(i / E) * kMaxE + i % E];
  for (int e = tid; e < E; e += blockDim.x) e2g_s[e] = c->expert_to_gpu[e];
  // QoS: the execution order of the experts by their summed priorities (identity without them)
  __shared__ float prio_s[kMaxE];
  if (kOrder) qos_order(c, priority != nullptr, prio_s);
  else __syncthreads();
  // 3. the plan
  if (tid < 32) harmony_warp(meta_s, G, E, e2g_s, c->eq_tokens, S_s, amt_s, le_s, amt32_s);
  __syncthreads();
  auto Sv = [&](int src, int e, int dst) { return S_s[(src * E + e) * G + dst]; };
  for (int i = tid; i < G * E * G; i += blockDim.x) {
    const int src = i / (E * G), e = (i / G) % E, dst = i % G;
    c->S[src][e][dst] = S_s[i];
  }
  // 4. tables from three prefix arrays (reusing meta_s, which is no longer needed):
  //    rin[dst][e]  = rows of expert e arriving at dst before expert e (exclusive prefix over e of
  //                   sum_src S[src][e][dst]) -> receive-buffer group starts of every rank;
  //    sout[src][dst] = rows src sends to destinations before dst (exclusive prefix over dst of
  //                   sum_e S[src][e][dst]) -> send-layout start of dst on src.
  __shared__ int32_t rin_s[kMaxG][kMaxE + 1];
  __shared__ int32_t sout_s[kMaxG][kMaxG];
  __syncthreads();
  if (tid < G) {  // one thread per destination rank: prefix over experts
    const int dst = tid;
    int r = 0;
    for (int e = 0; e < E; ++e) {
      rin_s[dst][e] = r;
      for (int s2 = 0; s2 < G; ++s2) r += Sv(s2, e, dst);
    }
    rin_s[dst][E] = r;
  } else if (tid >= 32 && tid < 32 + G) {  // one thread per source rank: prefix over destinations
    const int src = tid - 32;
    int r = 0;
    for (int d2 = 0; d2 < G; ++d2) {
      sout_s[src][d2] = r;
      for (int e2 = 0; e2 < E; ++e2) r += Sv(src, e2, d2);
    }
  }
  __syncthreads();
  for (int i = tid; i < E * G; i += blockDim.x) {
    const int e = i / G, dst = i % G;
    // sender side (this rank)
    int cs = 0;
    for (int d2 = 0; d2 <= dst; ++d2) cs += Sv(me, e, d2);
    c->cum_split[e][dst] = cs;
    int sb = sout_s[me][dst];
    for (int e2 = 0; e2 < e; ++e2) sb += Sv(me, e2, dst);
    c->send_base[e][dst] = sb;
    int rb = rin_s[dst][e];  // chunk (me, e) in dst's receive buffer: after lower sources
    for (int s2 = 0; s2 < me; ++s2) rb += Sv(s2, e, dst);
    c->remote_base[e][dst] = rb;
    // receiver side (this rank), chunk of source `src`
    const int src = dst;
    int cst = rin_s[me][e];
    for (int s2 = 0; s2 < src; ++s2) cst += Sv(s2, e, me);
    c->chunk_start[e][src] = cst;
    c->chunk_len[e][src] = Sv(src, e, me);
    int rs = sout_s[src][me];  // where that chunk goes back in src's send layout
    for (int e2 = 0; e2 < e; ++e2) rs += Sv(src, e2, me);
    c->ret_start[e][src] = rs;
  }
  for (int e = tid; e <= E; e += blockDim.x) c->group_offsets[e] = rin_s[me][e];
  if (tid == 0) {
    const int r = rin_s[me][E];
    c->recv_total = r;
    if (r > c->recv_capacity) record_error(err, kErrCapacity);
    int snd = 0;
    for (int e2 = 0; e2 < E; ++e2)
      for (int d2 = 0; d2 < G; ++d2) snd += Sv(me, e2, d2);
    if (snd > c->ret_capacity) record_error(err, kErrCapacity);
  }
  __syncthreads();
  if (tid == 0) {
    __threadfence();
    *reinterpret_cast<volatile uint32_t*>(&c->epoch) = epoch;
  }
}

// ------------------------------------------------------------------ dispatch kernel
// A resident grid (a few CTAs per SM): warp w copies the routed rows w, w + W, ... (W warps in
// the grid), each one row of d elements with eight 16-byte loads in flight per lane; the last
// CTA to finish raises the dispatch flag at every peer.  Few CTAs keep the per-CTA completion
// fence (system scope) rare.
template <int ESZ>
__global__ void __launch_bounds__(256) dispatch_kernel(dsca_ep_dispatch_args a, Ctx* c) {
  const int lane = threadIdx.x & 31;
  const int nwarps = (int)(gridDim.x * blockDim.x) >> 5;
  const int total = a.T * a.top_k;
  const int G = c->G;
  const size_t row_bytes = (size_t)a.d * ESZ;
  for (int w = (int)((blockIdx.x * blockDim.x + threadIdx.x) >> 5); w < total; w += nwarps) {
    const int t = w / a.top_k;
    const int e = a.topk_ids[w];
    bool ok = e >= 0 && e < c->E;
    int dst = 0, q = 0;
    if (ok) {
      q = a.block_base[(size_t)(t / DSCA_ROUTER_TOKENS) * c->E + e] + a.local_rank[w];
      while (dst < G && q >= c->cum_split[e][dst]) ++dst;
      ok = dst < G;
    }
    if (!ok) {
      if (lane == 0) record_error(a.err, kErrIndex);
      continue;
    }
    const int before = dst > 0 ? c->cum_split[e][dst - 1] : 0;
    const int rrow = c->remote_base[e][dst] + (q - before);
    const int srow = c->send_base[e][dst] + (q - before);
    if (rrow < 0 || rrow >= c->recv_capacity || srow < 0 || srow >= c->ret_capacity) {
      if (lane == 0) record_error(a.err, kErrCapacity);
      continue;
    }
    if (lane == 0) a.token_row[w] = srow;
    const uint4* src = reinterpret_cast<const uint4*>(reinterpret_cast<const char*>(a.x) + (size_t)t * row_bytes);
    uint4* dp = reinterpret_cast<uint4*>(c->recv[dst] + (size_t)rrow * row_bytes);
    if (ESZ == 2 && a.out_f16) {
      // bf16 -> f16 on the way (the operand of the fp8-weight FFN); the token's slot-0 warp also
      // writes the local f16 copy of x for the shared expert
      uint4* xh = (a.x_f16 != nullptr && (w % a.top_k) == 0)
                      ? reinterpret_cast<uint4*>(reinterpret_cast<char*>(a.x_f16) + (size_t)t * row_bytes)
                      : nullptr;
      for (int v = lane; v < (int)(row_bytes / 16); v += 32) {
        const uint4 o = bf16x8_to_f16x8(src[v]);
        dp[v] = o;
        if (xh != nullptr) xh[v] = o;
      }
    } else {
      warp_copy_row(dp, src, (int)(row_bytes / 16), lane);
    }
  }
  signal_when_grid_done(c, &c->dispatch_done, kDispatch);
}

// ------------------------------------------------------------------ return kernel
// Row r of this rank's receive layout (expert e, chunk of source src) goes to row
// ret_start[e][src] + (r - chunk_start[e][src]) of src's return buffer.  A resident grid: warp w
// takes rows w, w + W, ..., one row at a time (each NVLink store instruction writes 512
// contiguous bytes); the row count is read on the device.  The last CTA sets the return flags.
template <int ESZ>
__global__ void __launch_bounds__(256) return_kernel(Ctx* c, const char* y, int d, int32_t* err) {
  const int lane = threadIdx.x & 31;
  const int nwarps = (int)(gridDim.x * blockDim.x) >> 5;
  const int total = c->recv_total;
  for (int r = (int)((blockIdx.x * blockDim.x + threadIdx.x) >> 5); r < total; r += nwarps) {
    // expert: upper bound over group_offsets
    int lo = 0, hi = c->E;
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (c->group_offsets[mid] <= r) lo = mid; else hi = mid;
    }
    const int e = lo;
    char* dst = nullptr;
    for (int src = 0; src < c->G; ++src) {
      const int cs = c->chunk_start[e][src];
      if (r >= cs && r < cs + c->chunk_len[e][src]) {
        dst = c->ret[src] + (size_t)(c->ret_start[e][src] + r - cs) * d * ESZ;
        break;
      }
    }
    if (dst == nullptr) {
      if (lane == 0) record_error(err, kErrIndex);
      continue;
    }
    const uint4* s = reinterpret_cast<const uint4*>(y + (size_t)r * d * ESZ);
    warp_copy_row(reinterpret_cast<uint4*>(dst), s, d * ESZ / 16, lane);
  }
  signal_when_grid_done(c, &c->return_done, kReturn);
}

// ------------------------------------------------------------------ wait kernel
__global__ void wait_kernel(Ctx* c, int kind, uint64_t limit_ns, int32_t* err) {
  const int src = threadIdx.x;
  if (src < c->G) {
    const uint32_t epoch = *reinterpret_cast<volatile uint32_t*>(&c->epoch);
    if (!wait_flag(c->flags[c->me] + kind * kMaxG + src, epoch, limit_ns)) record_error(err, kErrWaitTimeout);
  }
}

// ------------------------------------------------------------------ test hook: device plan
__global__ void plan_eval_kernel(const int32_t* meta, int G, int E, const int32_t* e2g, int eq, int32_t* S) {
  __shared__ int32_t meta_s[kMaxG * kMaxE];
  __shared__ int32_t S_s[kMaxG * kMaxE * kMaxG];
  __shared__ long long amt_s[kMaxG];
  __shared__ int32_t amt32_s[kMaxG];
  __shared__ int32_t le_s[kMaxE * kMaxG];
  __shared__ int32_t e2g_s[kMaxE];
  for (int i = threadIdx.x; i < G * E; i += 32) meta_s[i] = meta[i];
  for (int i = threadIdx.x; i < E; i += 32) e2g_s[i] = e2g[i];
  __syncwarp();
  harmony_warp(meta_s, G, E, e2g_s, eq, S_s, amt_s, le_s, amt32_s);
  for (int i = threadIdx.x; i < G * E * G; i += 32) S[i] = S_s[i];
}

}  // namespace ep
}  // namespace dsca

// ------------------------------------------------------------------ C ABI
using dsca::ep::Ctx;
using dsca::ep::kMaxE;
using dsca::ep::kMaxG;

extern "C" {

size_t dsca_ep_ctx_bytes(void) { return sizeof(Ctx); }

int32_t* dsca_ep_group_offsets(void* ctx_dev) {
  return ctx_dev == nullptr ? nullptr : static_cast<Ctx*>(ctx_dev)->group_offsets;
}

int dsca_ep_read_plan(void* ctx_dev, int32_t* S_host, int32_t* recv_total_host, dsca_stream_t stream) {
  if (ctx_dev == nullptr || S_host == nullptr || recv_total_host == nullptr) return DSCA_ERR_BAD_ARG;
  Ctx* c = static_cast<Ctx*>(ctx_dev);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (cudaMemcpyAsync(S_host, c->S, sizeof(c->S), cudaMemcpyDeviceToHost, st) != cudaSuccess ||
      cudaMemcpyAsync(recv_total_host, &c->recv_total, sizeof(int32_t), cudaMemcpyDeviceToHost, st) != cudaSuccess)
    return DSCA_ERR_CUDA;
  return cudaStreamSynchronize(st) == cudaSuccess ? DSCA_OK : DSCA_ERR_CUDA;
}

int dsca_ep_init(void* ctx_dev, const dsca_ep_setup* s, dsca_stream_t stream) {
  if (ctx_dev == nullptr || s == nullptr || s->G <= 0 || s->G > kMaxG || s->E <= 0 || s->E > kMaxE || s->me < 0 ||
      s->me >= s->G || s->d <= 0 || s->expert_to_gpu == nullptr || s->recv_capacity <= 0 || s->ret_capacity <= 0)
    return DSCA_ERR_BAD_ARG;
  if (s->elem_bytes != 2 && s->elem_bytes != 4) return DSCA_ERR_BAD_ARG;
  static thread_local Ctx host;  // staging copy (stream-ordered H2D below is synchronised before return)
  memset(&host, 0, sizeof(Ctx));
  host.G = s->G;
  host.E = s->E;
  host.me = s->me;
  host.d = s->d;
  host.recv_capacity = s->recv_capacity;
  host.ret_capacity = s->ret_capacity;
  host.eq_tokens = s->eq_tokens;
  host.elem_bytes = s->elem_bytes;
  host.epoch = s->start_epoch;
  host.prio_epoch = s->start_epoch;
  for (int e = 0; e < s->E; ++e) {
    if (s->expert_to_gpu[e] < 0 || s->expert_to_gpu[e] >= s->G) return DSCA_ERR_BAD_ARG;
    host.expert_to_gpu[e] = s->expert_to_gpu[e];
  }
  for (int p = 0; p < s->G; ++p) {
    if (s->flags[p] == nullptr || s->meta[p] == nullptr || s->recv[p] == nullptr || s->ret[p] == nullptr)
      return DSCA_ERR_BAD_ARG;
    host.flags[p] = static_cast<uint32_t*>(s->flags[p]);
    host.meta[p] = static_cast<int32_t*>(s->meta[p]);
    host.recv[p] = static_cast<char*>(s->recv[p]);
    host.ret[p] = static_cast<char*>(s->ret[p]);
  }
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (cudaMemcpyAsync(ctx_dev, &host, sizeof(Ctx), cudaMemcpyHostToDevice, st) != cudaSuccess) return DSCA_ERR_CUDA;
  if (cudaStreamSynchronize(st) != cudaSuccess) return DSCA_ERR_CUDA;
  return DSCA_OK;
}

int32_t* dsca_ep_group_order(void* ctx_dev) {
  return ctx_dev == nullptr ? nullptr : static_cast<Ctx*>(ctx_dev)->group_order;
}

int dsca_ep_plan(void* ctx_dev, const int32_t* counts, const float* priority, uint64_t limit_ns, int32_t* err,
                 dsca_stream_t stream) {
  if (ctx_dev == nullptr || counts == nullptr) return DSCA_ERR_BAD_ARG;
  dsca::ep::plan_kernel<true><<<1, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      static_cast<Ctx*>(ctx_dev), counts, priority, limit_ns, err);
  return cudaGetLastError() == cudaSuccess ? DSCA_OK : DSCA_ERR_CUDA;
}

int dsca_ep_plan_counts(void* ctx_dev, const int32_t* counts, uint64_t limit_ns, int32_t* err, dsca_stream_t stream) {
  if (ctx_dev == nullptr || counts == nullptr) return DSCA_ERR_BAD_ARG;
  dsca::ep::plan_kernel<false><<<1, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      static_cast<Ctx*>(ctx_dev), counts, nullptr, limit_ns, err);
  return cudaGetLastError() == cudaSuccess ? DSCA_OK : DSCA_ERR_CUDA;
}

int dsca_ep_priority(void* ctx_dev, const float* priority, uint64_t limit_ns, int32_t* err, dsca_stream_t stream) {
  if (ctx_dev == nullptr || priority == nullptr) return DSCA_ERR_BAD_ARG;
  dsca::ep::priority_kernel<<<1, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(static_cast<Ctx*>(ctx_dev),
                                                                                priority, limit_ns, err);
  return cudaGetLastError() == cudaSuccess ? DSCA_OK : DSCA_ERR_CUDA;
}

int dsca_ep_dispatch(const dsca_ep_dispatch_args* a, dsca_stream_t stream) {
  if (a == nullptr || a->ctx == nullptr || a->x == nullptr || a->topk_ids == nullptr || a->local_rank == nullptr ||
      a->block_base == nullptr || a->token_row == nullptr || a->top_k <= 0 || a->top_k > DSCA_MAX_TOPK || a->T < 0)
    return DSCA_ERR_BAD_ARG;
  if (a->dtype != DSCA_BF16 && a->dtype != DSCA_F32) return DSCA_ERR_BAD_ARG;
  const int esz = a->dtype == DSCA_BF16 ? 2 : 4;
  if (((size_t)a->d * esz) % 16 != 0 || (reinterpret_cast<uintptr_t>(a->x) & 15u)) return DSCA_ERR_BAD_ARG;
  if (a->out_f16 && (a->dtype != DSCA_BF16 || (reinterpret_cast<uintptr_t>(a->x_f16) & 15u))) return DSCA_ERR_BAD_ARG;
  const long long warps = (long long)a->T * a->top_k;
  // >= 1 CTA so the flag is still set; at most kCtasPerSm resident CTAs per SM (grid-stride)
  const int sms = dsca::current_device_sms();
  if (sms == 0) return DSCA_ERR_CUDA;
  const long long need = warps > 0 ? (warps * 32 + 255) / 256 : 1;
  const int blocks = (int)std::min<long long>(need, (long long)dsca::ep::kCtasPerSm * sms);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (esz == 2)
    dsca::ep::dispatch_kernel<2><<<blocks, 256, 0, st>>>(*a, static_cast<Ctx*>(a->ctx));
  else
    dsca::ep::dispatch_kernel<4><<<blocks, 256, 0, st>>>(*a, static_cast<Ctx*>(a->ctx));
  return cudaGetLastError() == cudaSuccess ? DSCA_OK : DSCA_ERR_CUDA;
}

int dsca_ep_return(void* ctx_dev, const void* y, int d, int dtype, int max_rows, int32_t* err, dsca_stream_t stream) {
  if (ctx_dev == nullptr || y == nullptr || d <= 0 || max_rows < 0) return DSCA_ERR_BAD_ARG;
  if (dtype != DSCA_BF16 && dtype != DSCA_F32) return DSCA_ERR_BAD_ARG;
  const int esz = dtype == DSCA_BF16 ? 2 : 4;
  if (((size_t)d * esz) % 16 != 0 || (reinterpret_cast<uintptr_t>(y) & 15u)) return DSCA_ERR_BAD_ARG;
  // the row count is on the device: a resident grid (grid-stride over the rows) sized for at
  // most max_rows rows; >= 1 CTA so the flag is set
  const int sms = dsca::current_device_sms();
  if (sms == 0) return DSCA_ERR_CUDA;
  const long long need = std::max(1LL, ((long long)max_rows * 32 + 255) / 256);
  const int blocks = (int)std::min<long long>(need, (long long)dsca::ep::kCtasPerSm * sms);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (esz == 2)
    dsca::ep::return_kernel<2><<<blocks, 256, 0, st>>>(static_cast<Ctx*>(ctx_dev), static_cast<const char*>(y), d, err);
  else
    dsca::ep::return_kernel<4><<<blocks, 256, 0, st>>>(static_cast<Ctx*>(ctx_dev), static_cast<const char*>(y), d, err);
  return cudaGetLastError() == cudaSuccess ? DSCA_OK : DSCA_ERR_CUDA;
}

int dsca_ep_wait(void* ctx_dev, int kind, uint64_t limit_ns, int32_t* err, dsca_stream_t stream) {
  if (ctx_dev == nullptr || kind < 0 || kind > 2) return DSCA_ERR_BAD_ARG;
  dsca::ep::wait_kernel<<<1, 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>(static_cast<Ctx*>(ctx_dev), kind,
                                                                            limit_ns, err);
  return cudaGetLastError() == cudaSuccess ? DSCA_OK : DSCA_ERR_CUDA;
}

int dsca_ep_plan_eval(const int32_t* meta, int G, int E, const int32_t* expert_to_gpu, int eq_tokens, int32_t* S,
                      dsca_stream_t stream) {
  if (meta == nullptr || expert_to_gpu == nullptr || S == nullptr || G <= 0 || G > kMaxG || E <= 0 || E > kMaxE)
    return DSCA_ERR_BAD_ARG;
  dsca::ep::plan_eval_kernel<<<1, 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>(meta, G, E, expert_to_gpu,
                                                                                 eq_tokens, S);
  return cudaGetLastError() == cudaSuccess ? DSCA_OK : DSCA_ERR_CUDA;
}

// ------------------------------------------------------------------ the symmetric region itself
// Its own cudaMalloc allocation (set-up time, once per engine), zeroed, so that CUDA IPC maps
// exactly this region into the peers.
int dsca_ep_region_alloc(size_t bytes, void** ptr) {
  if (ptr == nullptr || bytes == 0) return DSCA_ERR_BAD_ARG;
  void* p = nullptr;
  if (cudaMalloc(&p, bytes) != cudaSuccess) return DSCA_ERR_CUDA;
  if (cudaMemset(p, 0, bytes) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess) {
    cudaFree(p);
    return DSCA_ERR_CUDA;
  }
  *ptr = p;
  return DSCA_OK;
}

int dsca_ep_region_free(void* ptr) {
  if (ptr == nullptr) return DSCA_ERR_BAD_ARG;
  return cudaFree(ptr) == cudaSuccess ? DSCA_OK : DSCA_ERR_CUDA;
}

// ------------------------------------------------------------------ CUDA IPC of the symmetric region
typedef CUresult (*PFN_getAddressRange)(CUdeviceptr*, size_t*, CUdeviceptr);

static PFN_getAddressRange get_range_fn() {
  static PFN_getAddressRange fn = nullptr;
  if (fn == nullptr) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return nullptr;
    fn = reinterpret_cast<PFN_getAddressRange>(p);
  }
  return fn;
}

int dsca_ipc_export(const void* ptr, void* handle64, size_t* offset) {
  if (ptr == nullptr || handle64 == nullptr || offset == nullptr) return DSCA_ERR_BAD_ARG;
  PFN_getAddressRange range = get_range_fn();
  if (range == nullptr) return DSCA_ERR_CUDA;
  CUdeviceptr base = 0;
  size_t size = 0;
  if (range(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS) return DSCA_ERR_CUDA;
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base)) != cudaSuccess) return DSCA_ERR_CUDA;
  static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handle size");
  memcpy(handle64, &h, 64);
  *offset = static_cast<size_t>(reinterpret_cast<CUdeviceptr>(ptr) - base);
  return DSCA_OK;
}

int dsca_ipc_import(const void* handle64, size_t offset, void** ptr) {
  if (handle64 == nullptr || ptr == nullptr) return DSCA_ERR_BAD_ARG;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle64, 64);
  void* base = nullptr;
  if (cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) return DSCA_ERR_CUDA;
  *ptr = static_cast<char*>(base) + offset;
  return DSCA_OK;
}

int dsca_ipc_close(void* ptr, size_t offset) {
  if (ptr == nullptr) return DSCA_ERR_BAD_ARG;
  return cudaIpcCloseMemHandle(static_cast<char*>(ptr) - offset) == cudaSuccess ? DSCA_OK : DSCA_ERR_CUDA;
}

}  // extern "C"
