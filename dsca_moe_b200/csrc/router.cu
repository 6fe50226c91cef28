// K1 — router: logits, softmax, top-1 / top-k, shared-expert gate, per-block histogram,
// in-block stable ranks and (optionally) the per-expert scan, fused in one launch.
//
// Reference semantics: Router.standard_forward (src/harmonymoe/router.py:52-63) and the
// argmax at src/qosmoe/moe_layer.py:287 for the Switch top-1 block; gate / softmax(fp32) /
// topk / renorm / cast of ShardedQwenMoE.forward (qwen_ep_adapter/qwen_ep.py:48-53) and the
// shared-expert gate sigmoid (qwen_ep.py:94) for the Qwen block.
//
// Fixed arithmetic order of a logit (the C oracle follows it bit for bit):
//   C = 32 * ceil(d / 256); chunk q covers i in [qC, min(d, (q+1)C)) (at most 8 chunks);
//   S_q = fma chain over the chunk in increasing i from 0.0f; logit = partials summed left to
//   right, rounded to the router dtype.
//
// Layout: one CTA = 32 tokens (DSCA_ROUTER_TOKENS) x 64 router rows (E experts, then the shared
// gate row, then zeros), 1024 threads = 8 chunk groups of 128.  In group q, thread g owns tokens
// 4*(g/16)..+3 and rows g%16 + 16j (j < 4): a 4 x 4 register tile fed by 16-byte shared-memory
// reads (x and W staged row-major in fp32, pitch 20 floats so the 16 row lanes of a warp hit
// distinct banks).  Each group streams its chunk in 16-wide k slices through two buffers,
// fetching the next slice into registers while computing the current one, and syncs on its own
// named barrier.  The chunk partials meet in shared memory; softmax and selection then run one
// warp per token.  With the fused scan, the last CTA to finish turns every block's histogram into
// the per-expert counts, offsets and block bases (stable: block order, then token order).
#include "common.cuh"

namespace dsca {
namespace router {

constexpr int kTokens = DSCA_ROUTER_TOKENS;  // 32
constexpr int kRows = 64;                    // router rows (E + shared gate <= 64)
constexpr int kGroups = 8;
constexpr int kGroupThreads = 128;
constexpr int kThreads = kGroups * kGroupThreads;  // 1024
constexpr int kKS = 16;                      // k slice
constexpr int kP = kKS + 4;                  // staging row pitch (floats)
constexpr int kStageFloats = kTokens * kP + kRows * kP;
constexpr int kLP = kRows + 1;               // logit tile pitch
constexpr size_t kSmemBytes = sizeof(float) * (size_t)(kGroups * 2 * kStageFloats);

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
};

__device__ __forceinline__ void group_sync(int q) {
  asm volatile("bar.sync %0, %1;" ::"r"(q + 1), "r"(kGroupThreads) : "memory");
}

// Row pointer of router row r (router weight, shared-gate row, or nothing).
template <typename T>
__device__ __forceinline__ const T* wrow(const Args& a, int r) {
  if (r < a.E) return reinterpret_cast<const T*>(a.w_router) + (size_t)r * a.d;
  if (r == a.E && a.w_shared_gate != nullptr) return reinterpret_cast<const T*>(a.w_shared_gate);
  return nullptr;
}

// Per-thread staging registers for one 16-wide k slice of the group's chunk.
template <typename T>
struct Slice;

template <>
struct Slice<__nv_bfloat16> {
  // x: 32 tokens x 16 k = 64 x uint4 (threads 0..63); W: 64 rows x 16 k = 128 x uint4 (one each)
  uint4 xv, wv;
  __device__ void fetch(const Args& a, int g, int tok0, int k0, int kend) {
    const __nv_bfloat16* x = reinterpret_cast<const __nv_bfloat16*>(a.x);
    xv = make_uint4(0, 0, 0, 0);
    if (g < 64) {
      const int t = g >> 1, c = (g & 1) * 8;
      if (tok0 + t < a.T && k0 + c < kend) xv = *reinterpret_cast<const uint4*>(x + (size_t)(tok0 + t) * a.d + k0 + c);
    }
    const int r = g >> 1, c = (g & 1) * 8;
    const __nv_bfloat16* w = wrow<__nv_bfloat16>(a, r);
    wv = make_uint4(0, 0, 0, 0);
    if (w != nullptr && k0 + c < kend) wv = *reinterpret_cast<const uint4*>(w + k0 + c);
  }
  static __device__ void put8(float* dst, const uint4& u) {
    const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(&u);
    *reinterpret_cast<float4*>(dst) = make_float4(__bfloat162float(h[0]), __bfloat162float(h[1]),
                                                  __bfloat162float(h[2]), __bfloat162float(h[3]));
    *reinterpret_cast<float4*>(dst + 4) = make_float4(__bfloat162float(h[4]), __bfloat162float(h[5]),
                                                      __bfloat162float(h[6]), __bfloat162float(h[7]));
  }
  __device__ void store(float* xs, float* ws, int g) const {
    if (g < 64) put8(xs + (g >> 1) * kP + (g & 1) * 8, xv);
    put8(ws + (g >> 1) * kP + (g & 1) * 8, wv);
  }
};

template <>
struct Slice<float> {
  // x: 32 x 16 floats = 128 float4 (one each); W: 64 x 16 = 256 float4 (two each)
  float4 xv, wv[2];
  __device__ void fetch(const Args& a, int g, int tok0, int k0, int kend) {
    const float* x = reinterpret_cast<const float*>(a.x);
    {
      const int t = g >> 2, c = (g & 3) * 4;
      xv = make_float4(0.f, 0.f, 0.f, 0.f);
      if (tok0 + t < a.T && k0 + c < kend) xv = *reinterpret_cast<const float4*>(x + (size_t)(tok0 + t) * a.d + k0 + c);
    }
#pragma unroll
    for (int v = 0; v < 2; ++v) {
      const int idx = g + v * kGroupThreads;
      const int r = idx >> 2, c = (idx & 3) * 4;
      const float* w = wrow<float>(a, r);
      wv[v] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (w != nullptr && k0 + c < kend) wv[v] = *reinterpret_cast<const float4*>(w + k0 + c);
    }
  }
  __device__ void store(float* xs, float* ws, int g) const {
    *reinterpret_cast<float4*>(xs + (g >> 2) * kP + (g & 3) * 4) = xv;
#pragma unroll
    for (int v = 0; v < 2; ++v) {
      const int idx = g + v * kGroupThreads;
      *reinterpret_cast<float4*>(ws + (idx >> 2) * kP + (idx & 3) * 4) = wv[v];
    }
  }
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

// Per-expert counts, offsets and block bases from all blocks' histograms (one CTA).
__device__ void scan_blocks(const Args& a, int nb, int* cnt_s) {
  const int E = a.E;
  const volatile int32_t* hist = a.block_hist;
  // thread (e, c): a contiguous run of blocks of expert e; 16 runs per expert
  constexpr int kRuns = 16;
  __shared__ int part[kRows][kRuns + 1];
  const int per = (nb + kRuns - 1) / kRuns;
  for (int base_e = 0; base_e < E; base_e += kThreads / kRuns) {
    const int e = base_e + threadIdx.x / kRuns, c = threadIdx.x % kRuns;
    const int b0 = c * per, b1 = min(nb, b0 + per);
    int s = 0;
    if (e < E)
      for (int b = b0; b < b1; ++b) s += hist[(size_t)b * E + e];
    if (e < E) part[e][c] = s;
    __syncthreads();
    if (e < E && c == 0) {
      int run = 0;
      for (int i = 0; i < kRuns; ++i) {
        const int v = part[e][i];
        part[e][i] = run;
        run += v;
      }
      cnt_s[e] = run;
      a.counts[e] = run;
    }
    __syncthreads();
    if (e < E) {
      int run = part[e][c];
      for (int b = b0; b < b1; ++b) {
        const int v = hist[(size_t)b * E + e];
        a.block_base[(size_t)b * E + e] = run;
        run += v;
      }
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    int run = 0;
    for (int e = 0; e < E; ++e) {
      a.offsets[e] = run;
      run += cnt_s[e];
    }
    a.offsets[E] = run;
  }
}

template <typename T>
__global__ void __launch_bounds__(kThreads, 1) router_kernel(Args a) {
  extern __shared__ __align__(16) float smem[];
  __shared__ float lg_s[kTokens * kLP];
  __shared__ int ids_s[kTokens][DSCA_MAX_TOPK];
  __shared__ int cnt_s[kRows];
  __shared__ int is_last;

  const int tid = threadIdx.x;
  const int q = tid / kGroupThreads;  // chunk group
  const int g = tid % kGroupThreads;
  const int tok0 = blockIdx.x * kTokens;
  const int E = a.E;
  const bool has_sg = a.w_shared_gate != nullptr;
  const bool tau_bf16 = sizeof(T) == 2;

  // ---------------- chunk partial sums: 4 x 4 tile per thread
  const int C = 32 * ((a.d + 255) / 256);
  const int nq = (a.d + C - 1) / C;
  const int kbeg = q * C, kend = min(a.d, kbeg + C);
  const int tq = g >> 4, rq = g & 15;
  float acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.0f;

  float* stage0 = smem + q * 2 * kStageFloats;
  if (q < nq) {
    Slice<T> sl;
    sl.fetch(a, g, tok0, kbeg, kend);
    sl.store(stage0, stage0 + kTokens * kP, g);
    group_sync(q);
    int s = 0;
    for (int k0 = kbeg; k0 < kend; k0 += kKS, s ^= 1) {
      const bool more = k0 + kKS < kend;
      if (more) sl.fetch(a, g, tok0, k0 + kKS, kend);  // in flight during the compute below
      const float* xs = stage0 + s * kStageFloats;
      const float* xb = xs + (4 * tq) * kP;
      const float* wb = xs + kTokens * kP + rq * kP;
      const int kmax = min(kKS, kend - k0);  // a multiple of 8 (bf16) or 4 (fp32)
      for (int k = 0; k < kmax; k += 4) {
        float4 xv[4], wv[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) xv[i] = *reinterpret_cast<const float4*>(xb + i * kP + k);
#pragma unroll
        for (int j = 0; j < 4; ++j) wv[j] = *reinterpret_cast<const float4*>(wb + 16 * j * kP + k);
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            acc[i][j] = __fmaf_rn(xv[i].x, wv[j].x, acc[i][j]);
            acc[i][j] = __fmaf_rn(xv[i].y, wv[j].y, acc[i][j]);
            acc[i][j] = __fmaf_rn(xv[i].z, wv[j].z, acc[i][j]);
            acc[i][j] = __fmaf_rn(xv[i].w, wv[j].w, acc[i][j]);
          }
      }
      if (more) {
        float* nx = stage0 + (s ^ 1) * kStageFloats;  // last read two slices ago
        sl.store(nx, nx + kTokens * kP, g);
      }
      group_sync(q);
    }
  }
  __syncthreads();  // staging buffers are reused for the partials below
  float* part = smem;  // [nq][32 tokens][64 rows]
  if (q < nq) {
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) part[(q * kTokens + 4 * tq + i) * kRows + rq + 16 * j] = acc[i][j];
  }
  __syncthreads();
  for (int idx = tid; idx < kTokens * kRows; idx += kThreads) {
    const int t = idx / kRows, r = idx % kRows;
    float tot = part[t * kRows + r];
    for (int qq = 1; qq < nq; ++qq) tot = __fadd_rn(tot, part[(qq * kTokens + t) * kRows + r]);
    lg_s[t * kLP + r] = tau_bf16 ? round_bf16(tot) : tot;
  }
  __syncthreads();

  // ---------------- softmax and selection: one warp per token
  const int warp = tid >> 5, lane = tid & 31;
  const int e0 = lane, e1 = lane + 32;
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
    float m = fmaxf((e0 < E) ? l0 : -INFINITY, (e1 < E) ? l1 : -INFINITY);
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
    const float x0 = (e0 < E) ? exp_neg(__fsub_rn(l0, m)) : 0.0f;
    const float x1 = (e1 < E) ? exp_neg(__fsub_rn(l1, m)) : 0.0f;
    float ps = (e0 < E) ? __fadd_rn(0.0f, x0) : 0.0f;
    if (e1 < E) ps = __fadd_rn(ps, x1);
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) ps = __fadd_rn(ps, __shfl_xor_sync(0xffffffffu, ps, off));
    float p0 = (e0 < E) ? __fdiv_rn(x0, ps) : -INFINITY;
    float p1 = (e1 < E) ? __fdiv_rn(x1, ps) : -INFINITY;

    if (a.mode == DSCA_ROUTE_SWITCH_TOP1) {
      if (tau_bf16) {
        p0 = (e0 < E) ? round_bf16(p0) : -INFINITY;
        p1 = (e1 < E) ? round_bf16(p1) : -INFINITY;
      }
      float bv = p0;
      int bi = e0;
      if (p1 > bv) { bv = p1; bi = e1; }
#pragma unroll
      for (int off = 16; off >= 1; off >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
        if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
      }
      if (lane == 0) {
        ids_s[tl][0] = valid ? bi : -1;
        if (valid) {
          a.topk_ids[t] = bi;
          a.topk_w[t] = bv;
          if (a.expert_index != nullptr) a.expert_index[t] = bi;
        }
      }
    } else {
      bool taken0 = !(e0 < E), taken1 = !(e1 < E);
      float sel[DSCA_MAX_TOPK];
      int seli[DSCA_MAX_TOPK];
      for (int j = 0; j < a.top_k; ++j) {
        float bv = -INFINITY;
        int bi = 1 << 30;
        if (!taken0) { bv = p0; bi = e0; }
        if (!taken1 && (p1 > bv || bi == (1 << 30))) { bv = p1; bi = e1; }
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) {
          const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
          const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
          if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
        }
        if (bi == e0) taken0 = true;
        if (bi == e1) taken1 = true;
        sel[j] = bv;
        seli[j] = bi;
      }
      if (lane == 0) {
        float sum = 0.0f;
        if (a.norm_topk)
          for (int j = 0; j < a.top_k; ++j) sum = __fadd_rn(sum, sel[j]);
        for (int j = 0; j < a.top_k; ++j) {
          ids_s[tl][j] = valid ? seli[j] : -1;
          if (valid) {
            float w = a.norm_topk ? __fdiv_rn(sel[j], sum) : sel[j];
            if (a.weight_round_bf16) w = round_bf16(w);
            a.topk_ids[(size_t)t * a.top_k + j] = seli[j];
            a.topk_w[(size_t)t * a.top_k + j] = w;
          }
        }
        if (valid && a.expert_index != nullptr) a.expert_index[t] = seli[0];
      }
    }
  }
  __syncthreads();

  // ---------------- per-block histogram and stable in-block ranks (token, then slot order)
  const int k = (a.mode == DSCA_ROUTE_SWITCH_TOP1) ? 1 : a.top_k;
  for (int e = tid; e < E; e += kThreads) {
    int c = 0;
    for (int tl = 0; tl < kTokens; ++tl)
      for (int j = 0; j < k; ++j) c += (ids_s[tl][j] == e);
    a.block_hist[(size_t)blockIdx.x * E + e] = c;
  }
  for (int idx = tid; idx < kTokens * k; idx += kThreads) {
    const int tl = idx / k, j = idx % k;
    const int t = tok0 + tl;
    const int e = ids_s[tl][j];
    if (t >= a.T || e < 0) continue;
    int r = 0;
    for (int u = 0; u < tl; ++u)
      for (int jj = 0; jj < k; ++jj) r += (ids_s[u][jj] == e);
    a.local_rank[(size_t)t * k + j] = r;
  }

  // ---------------- fused scan: the last CTA to finish
  if (a.done_counter != nullptr) {
    __threadfence();
    __syncthreads();
    if (tid == 0) {
      const uint32_t prev = atomicAdd(a.done_counter, 1u);
      is_last = prev == gridDim.x - 1;
    }
    __syncthreads();
    if (is_last) {
      __threadfence();
      scan_blocks(a, gridDim.x, cnt_s);
      if (tid == 0) *a.done_counter = 0u;  // ready for the next launch (stream ordered)
    }
  }
}

}  // namespace router

int launch_router(const dsca_router_args* p, cudaStream_t stream) {
  static bool attr_done[2] = {false, false};
  router::Args a;
  a.x = p->x;
  a.w_router = p->w_router;
  a.w_shared_gate = p->w_shared_gate;
  a.T = p->T;
  a.d = p->d;
  a.E = p->E;
  a.top_k = p->mode == DSCA_ROUTE_SWITCH_TOP1 ? 1 : p->top_k;
  a.mode = p->mode;
  a.norm_topk = p->norm_topk;
  a.weight_round_bf16 = p->weight_round_bf16;
  a.logits = p->logits;
  a.topk_ids = p->topk_ids;
  a.topk_w = p->topk_w;
  a.expert_index = p->expert_index;
  a.shared_gate = p->shared_gate;
  a.block_hist = p->block_hist;
  a.local_rank = p->local_rank;
  const bool fused = p->done_counter != nullptr && p->counts != nullptr && p->offsets != nullptr &&
                     p->block_base != nullptr;
  a.counts = fused ? p->counts : nullptr;
  a.offsets = fused ? p->offsets : nullptr;
  a.block_base = fused ? p->block_base : nullptr;
  a.done_counter = fused ? p->done_counter : nullptr;
  const int nblocks = (p->T + router::kTokens - 1) / router::kTokens;
  cudaError_t e = cudaSuccess;
  if (p->dtype == DSCA_BF16) {
    if (!attr_done[0]) {
      e = cudaFuncSetAttribute(router::router_kernel<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               (int)router::kSmemBytes);
      attr_done[0] = e == cudaSuccess;
    }
    if (e == cudaSuccess)
      router::router_kernel<__nv_bfloat16><<<nblocks, router::kThreads, router::kSmemBytes, stream>>>(a);
  } else {
    if (!attr_done[1]) {
      e = cudaFuncSetAttribute(router::router_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               (int)router::kSmemBytes);
      attr_done[1] = e == cudaSuccess;
    }
    if (e == cudaSuccess) router::router_kernel<float><<<nblocks, router::kThreads, router::kSmemBytes, stream>>>(a);
  }
  if (e != cudaSuccess) return DSCA_ERR_CUDA;
  return cudaGetLastError() == cudaSuccess ? DSCA_OK : DSCA_ERR_CUDA;
}

// ------------------------------------------------------------------ exp test hook
__global__ void exp_neg_eval_kernel(const float* x, float* y, int n) {
  int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) y[i] = exp_neg(x[i]);
}

int launch_exp_eval(const float* x, float* y, int n, cudaStream_t stream) {
  if (n <= 0) return DSCA_OK;
  exp_neg_eval_kernel<<<(n + 255) / 256, 256, 0, stream>>>(x, y, n);
  return cudaGetLastError() == cudaSuccess ? DSCA_OK : DSCA_ERR_CUDA;
}

}  // namespace dsca
