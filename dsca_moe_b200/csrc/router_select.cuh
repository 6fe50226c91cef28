// K1 selection stage shared by the router kernels (router.cu: CUDA-core logits; router_tc.cu:
// tensor-core logits): from one 32-token block's logits in shared memory to the softmax, the
// top-1 / top-k choices and weights, the shared-expert gate, the block's per-expert histogram and
// in-block ranks, and (optionally) the fused scan run by the last CTA of the grid.  One CTA per
// 32-token block, kThreads threads; block b of the grid covers tokens [32 b, 32 b + 32).
//
// Reference semantics: Router.standard_forward (src/harmonymoe/router.py:52-63) and the argmax at
// src/qosmoe/moe_layer.py:287 for the Switch top-1 block; softmax(fp32) / topk / renorm / cast of
// ShardedQwenMoE.forward (qwen_ep_adapter/qwen_ep.py:48-53) and the shared-expert gate sigmoid
// (qwen_ep.py:94) for the Qwen block.
#pragma once

#include "common.cuh"

namespace dsca {
namespace router {

constexpr int kTokens = DSCA_ROUTER_TOKENS;  // 32
constexpr int kRows = 64;                    // router rows (E + shared gate <= 64)
constexpr int kThreads = 512;                // threads of a router CTA
constexpr int kLP = kRows + 1;               // logit tile pitch

struct Args {
  const void* x;
  const void* w_router;
  const void* w_shared_gate;
  int T, d, E, top_k, mode, norm_topk, weight_round_bf16;
  void* logits;
  int32_t* topk_ids;
  float* topk_w;
  int64_t* expert_index;
  float* shared_gate;
  int32_t* block_hist;
  int32_t* local_rank;
  int32_t* counts;
  int32_t* offsets;
  int32_t* block_base;
  uint32_t* done_counter;
  // precomputed logits [T][64] (fp32 values already rounded to the router dtype, rows past E
  // unused), or null: the kernel computes them (the chunked fp32 order below)
  const float* logits_in;
  int32_t* first_counts;  // += first-choice counts of the block's tokens, or null
};

template <typename T>
__device__ __forceinline__ void store_logit(void* logits, size_t i, float v);
template <>
__device__ __forceinline__ void store_logit<__nv_bfloat16>(void* logits, size_t i, float v) {
  reinterpret_cast<__nv_bfloat16*>(logits)[i] = __float2bfloat16_rn(v);
}
template <>
__device__ __forceinline__ void store_logit<float>(void* logits, size_t i, float v) {
  reinterpret_cast<float*>(logits)[i] = v;
}

// Order-preserving map of a (non-NaN) float onto uint32, and back.
__device__ __forceinline__ uint32_t ord_key(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float ord_val(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}


// Per-expert counts, offsets and block bases from all blocks' histograms (the last CTA).
// Thread (c, e) (e = tid % 64, c = tid / 64) takes a run of kR consecutive rows of column e per
// round of 8 kR rows: its kR loads go out together into registers (a warp reads 32 consecutive
// columns of one row per load), the 8 run sums of a column give each run its base, and each
// thread writes its rows' block bases from its registers.  Integer sums: the result does not
// depend on the order.
__device__ __forceinline__ void scan_blocks(const Args& a, int nb, int* run_s, int (*seg)[kRows]) {
  constexpr int kSegs = kThreads / kRows;  // 8
  constexpr int kR = 16;                   // rows per thread per round
  const int E = a.E, tid = threadIdx.x;
  const int e = tid % kRows, c = tid / kRows;
  if (tid < kRows) run_s[tid] = 0;
  __syncthreads();
  for (int b0 = 0; b0 < nb; b0 += kSegs * kR) {
    const int r0 = b0 + c * kR;
    int v[kR];
#pragma unroll
    for (int i = 0; i < kR; ++i) {
      const int r = r0 + i;
      v[i] = (e < E && r < nb) ? __ldcg(a.block_hist + (size_t)r * E + e) : 0;
    }
    int sum = 0;
#pragma unroll
    for (int i = 0; i < kR; ++i) sum += v[i];
    seg[c][e] = sum;
    __syncthreads();
    if (e < E) {
      int base = run_s[e];
      for (int cc = 0; cc < c; ++cc) base += seg[cc][e];
#pragma unroll
      for (int i = 0; i < kR; ++i) {
        const int r = r0 + i;
        if (r < nb) a.block_base[(size_t)r * E + e] = base;
        base += v[i];
      }
    }
    __syncthreads();
    if (c == 0 && e < E) {
      int tot = run_s[e];
      for (int cc = 0; cc < kSegs; ++cc) tot += seg[cc][e];
      run_s[e] = tot;
    }
    __syncthreads();
  }
  // counts, and offsets by a warp-wide scan (lane L holds experts L and L + 32)
  if (tid < 32) {
    const int L = tid;
    const int v0 = L < E ? run_s[L] : 0, v1 = L + 32 < E ? run_s[L + 32] : 0;
    int i0 = v0, i1 = v1;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int u0 = __shfl_up_sync(0xffffffffu, i0, off), u1 = __shfl_up_sync(0xffffffffu, i1, off);
      if (L >= off) { i0 += u0; i1 += u1; }
    }
    const int tot0 = __shfl_sync(0xffffffffu, i0, 31), tot1 = __shfl_sync(0xffffffffu, i1, 31);
    if (L < E) { a.counts[L] = v0; a.offsets[L] = i0 - v0; }
    if (L + 32 < E) { a.counts[L + 32] = v1; a.offsets[L + 32] = tot0 + i1 - v1; }
    if (L == 0) a.offsets[E] = tot0 + tot1;
  }
}

// Selection, histogram, ranks and the fused scan for block `block` (tokens [32 block, +32)).
// lg_s holds the block's logits [32][kLP] already rounded to the router dtype T; emask is zeroed
// and a __syncthreads() has passed since.  nblocks = ceil(T / 32) (blocks from nblocks on write
// no histogram row); the fused scan runs in the last of the grid's `ncta` CTAs to arrive.  Every
// thread of the CTA calls it.
template <typename T>
__device__ __forceinline__ void select_block(const Args& a, const float* lg_s, int (*ids_s)[DSCA_MAX_TOPK],
                                             uint32_t* emask, int* run_s, int (*seg_s)[kRows], int* is_last,
                                             int block, int nblocks, int ncta) {
  const int tid = threadIdx.x;
  const int tok0 = block * kTokens;
  const int E = a.E;
  const bool has_sg = a.w_shared_gate != nullptr;
  const bool tau_bf16 = sizeof(T) == 2;
  // ---------------- softmax and selection: one warp per token
  const int warp = tid >> 5, lane = tid & 31;
  const int e0 = lane, e1 = lane + 32;
  const int k = (a.mode == DSCA_ROUTE_SWITCH_TOP1) ? 1 : a.top_k;
  for (int tl = warp; tl < kTokens; tl += kThreads / 32) {
    const int t = tok0 + tl;
    const bool valid = t < a.T;
    const float l0 = lg_s[tl * kLP + e0];
    const float l1 = lg_s[tl * kLP + e1];
    if (valid) {
      if (e0 < E) store_logit<T>(a.logits, (size_t)t * E + e0, l0);
      if (e1 < E) store_logit<T>(a.logits, (size_t)t * E + e1, l1);
      if (has_sg && a.shared_gate != nullptr && (e0 == E || e1 == E)) {
        const float z = (e0 == E) ? l0 : l1;
        a.shared_gate[t] = 1.0f / (1.0f + expf(-z));
      }
    }
    // row max through an order-preserving integer key (one warp reduction)
    const uint32_t mkey = __reduce_max_sync(0xffffffffu, max((e0 < E) ? ord_key(l0) : 0u, (e1 < E) ? ord_key(l1) : 0u));
    const float m = ord_val(mkey);
    const float x0 = (e0 < E) ? exp_neg(__fsub_rn(l0, m)) : 0.0f;
    const float x1 = (e1 < E) ? exp_neg(__fsub_rn(l1, m)) : 0.0f;
    float ps = (e0 < E) ? __fadd_rn(0.0f, x0) : 0.0f;
    if (e1 < E) ps = __fadd_rn(ps, x1);
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) ps = __fadd_rn(ps, __shfl_xor_sync(0xffffffffu, ps, off));
    float p0 = (e0 < E) ? __fdiv_rn(x0, ps) : 0.0f;
    float p1 = (e1 < E) ? __fdiv_rn(x1, ps) : 0.0f;
    if (a.mode == DSCA_ROUTE_SWITCH_TOP1 && tau_bf16) {
      p0 = round_bf16(p0);
      p1 = round_bf16(p1);
    }

    // k rounds of (probability desc, expert id asc): probabilities are >= +0, so their bits
    // order like the values; key = bits + 1, 0 = no candidate.  Lane j keeps the j-th choice;
    // every lane sums the choices in rank order.
    float my_p = 0.0f, sum = 0.0f;
    int my_id = -1;
    bool taken0 = !(e0 < E), taken1 = !(e1 < E);
    for (int j = 0; j < k; ++j) {
      const uint32_t k0 = taken0 ? 0u : __float_as_uint(p0) + 1u;
      const uint32_t k1 = taken1 ? 0u : __float_as_uint(p1) + 1u;
      const uint32_t best = __reduce_max_sync(0xffffffffu, max(k0, k1));
      const uint32_t cand = (k0 == best) ? (uint32_t)e0 : ((k1 == best) ? (uint32_t)e1 : 0xffffffffu);
      const int bi = (int)__reduce_min_sync(0xffffffffu, cand);
      const float bv = __uint_as_float(best - 1u);
      if (bi == e0) taken0 = true;
      if (bi == e1) taken1 = true;
      if (lane == j) { my_p = bv; my_id = bi; }
      sum = __fadd_rn(sum, bv);
    }
    if (lane < k) {
      ids_s[tl][lane] = valid ? my_id : -1;
      if (valid) {
        float w = my_p;
        if (a.mode != DSCA_ROUTE_SWITCH_TOP1) {
          if (a.norm_topk) w = __fdiv_rn(my_p, sum);
          if (a.weight_round_bf16) w = round_bf16(w);
        }
        a.topk_ids[(size_t)t * k + lane] = my_id;
        a.topk_w[(size_t)t * k + lane] = w;
        if (lane == 0 && a.expert_index != nullptr) a.expert_index[t] = my_id;
        atomicOr(&emask[my_id], 1u << tl);
      }
    }
  }
  __syncthreads();

  // ---------------- per-block histogram and stable in-block ranks (token, then slot order):
  // an expert appears at most once per token, so the rank of (t, j) is the number of earlier
  // tokens of the block routed to the same expert
  for (int e = tid; e < E && block < nblocks; e += kThreads) {
    a.block_hist[(size_t)block * E + e] = __popc(emask[e]);
    if (a.done_counter != nullptr) __threadfence();  // the histogram before this CTA's arrival
  }
  // first-choice counts (the QoS planner's n(e)): integer atomics, one per expert of the block
  if (a.first_counts != nullptr)
    for (int e = tid; e < E && block < nblocks; e += kThreads) {
      int n = 0;
      for (int tl = 0; tl < kTokens; ++tl) n += ids_s[tl][0] == e ? 1 : 0;
      if (n) atomicAdd(&a.first_counts[e], n);
    }
  for (int idx = tid; idx < kTokens * k; idx += kThreads) {
    const int tl = idx / k, j = idx % k;
    const int t = tok0 + tl;
    const int e = ids_s[tl][j];
    if (t >= a.T || e < 0) continue;
    a.local_rank[(size_t)t * k + j] = __popc(emask[e] & ((1u << tl) - 1u));
  }

  // ---------------- fused scan: the last CTA to finish
  if (a.done_counter != nullptr) {
    __syncthreads();
    if (tid == 0) {
      const uint32_t prev = atomicAdd(a.done_counter, 1u);
      *is_last = prev == (uint32_t)ncta - 1u;
      __threadfence();
    }
    __syncthreads();
    if (*is_last) {
      scan_blocks(a, nblocks, run_s, seg_s);
      if (tid == 0) *a.done_counter = 0u;  // ready for the next launch (stream ordered)
    }
  }
}

// Kernel arguments from the C-ABI struct (logits_in left null).  The fused scan is on when all
// four of its outputs are set.
inline void fill_args(const dsca_router_args* p, Args* a) {
  a->logits_in = nullptr;
  a->x = p->x;
  a->w_router = p->w_router;
  a->w_shared_gate = p->w_shared_gate;
  a->T = p->T;
  a->d = p->d;
  a->E = p->E;
  a->top_k = p->mode == DSCA_ROUTE_SWITCH_TOP1 ? 1 : p->top_k;
  a->mode = p->mode;
  a->norm_topk = p->norm_topk;
  a->weight_round_bf16 = p->weight_round_bf16;
  a->logits = p->logits;
  a->topk_ids = p->topk_ids;
  a->topk_w = p->topk_w;
  a->expert_index = p->expert_index;
  a->shared_gate = p->shared_gate;
  a->block_hist = p->block_hist;
  a->local_rank = p->local_rank;
  const bool fused = p->done_counter != nullptr && p->counts != nullptr && p->offsets != nullptr &&
                     p->block_base != nullptr;
  a->counts = fused ? p->counts : nullptr;
  a->offsets = fused ? p->offsets : nullptr;
  a->block_base = fused ? p->block_base : nullptr;
  a->done_counter = fused ? p->done_counter : nullptr;
  a->first_counts = p->first_counts;
}

}  // namespace router
}  // namespace dsca
