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
// gate row, then zeros), 512 threads = 4 groups of 128.  Group j runs the chunks 2j and 2j+1
// side by side: every accumulator is a packed fp32x2 pair {S_2j, S_2j+1} of one (token, row),
// updated by __ffma2_rn, which rounds each element exactly like fmaf, so each element is its own
// chunk's fma chain.  A 16-wide k slice of both chunks is staged in shared memory interleaved
// ([t][k] -> {x[2jC + k], x[(2j+1)C + k]}, the same for W rows), so one 16-byte read gives two k
// of a pair.  Thread g owns tokens tq + 8i and rows rq + 16j (i, j < 4), a 4 x 4 tile of pairs;
// a warp spans 4 tq x 8 rq, arranged so that each group of 4 consecutive lanes covers 2 tq x 2 rq:
// a 16-byte shared-memory read then costs the minimum of two wavefronts (a lane quad receives
// one distinct 16-byte word per wavefront; the row pitch of 36 floats puts consecutive rows in
// distinct bank groups).  A shorter
// (or missing) second chunk reads zeros past its end: fma(0, 0, s) == s for every s such a chain
// can hold (it starts at +0.0f and never becomes -0.0f).  Each group streams its chunks through
// two buffers, fetching the next slice into registers while computing the current one, and
// syncs on its own named barrier.  The chunk partials meet in shared memory; softmax and
// selection then run one warp per token.  Per-block histograms and in-block ranks come from
// 32-bit token masks per expert.  With the fused scan, the last CTA to finish turns every
// block's histogram into the per-expert counts, offsets and block bases (stable: block order,
// then token order).
#include "router_select.cuh"

namespace dsca {
namespace router {

constexpr int kGroups = 4;                   // chunk pairs
constexpr int kGroupThreads = 128;
static_assert(kGroups * kGroupThreads == kThreads, "512 threads per router CTA");
constexpr int kKS = 16;                      // k slice (per chunk)
constexpr int kXP = 2 * kKS + 4;             // floats per token row of the interleaved x slice
constexpr int kWP = 2 * kKS + 4;             // floats per router row of the interleaved W slice
constexpr int kStageFloats = kTokens * kXP + kRows * kWP;
constexpr size_t kSmemBytes = sizeof(float) * (size_t)(kGroups * 2 * kStageFloats);
static_assert(kSmemBytes >= sizeof(float) * 8 * kTokens * kRows, "partials fit the staging area");


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

__device__ __forceinline__ void st4(float* p, float a, float b, float c, float d) {
  *reinterpret_cast<float4*>(p) = make_float4(a, b, c, d);
}

// Staging of one slice: 96 rows (32 tokens, then 64 router rows) x kKS/4 k-quads, kTasks per
// thread (task = g + 128 u).  A task reads 4 k of its row from each chunk of the pair and
// writes them interleaved.
constexpr int kQuads = kKS / 4;
constexpr int kTasks = (kTokens + kRows) * kQuads / kGroupThreads;
static_assert((kTokens + kRows) * kQuads % kGroupThreads == 0 && kGroupThreads % kQuads == 0, "task split");

template <typename T>
struct Vec4;  // 4 elements of T
template <>
struct Vec4<__nv_bfloat16> {
  using type = uint2;
  static __device__ type zero() { return make_uint2(0, 0); }
  static __device__ float lo(uint32_t u) { return __uint_as_float(u << 16); }
  static __device__ float hi(uint32_t u) { return __uint_as_float(u & 0xffff0000u); }
  static __device__ float4 f32(type v) { return make_float4(lo(v.x), hi(v.x), lo(v.y), hi(v.y)); }
};
template <>
struct Vec4<float> {
  using type = float4;
  static __device__ type zero() { return make_float4(0.f, 0.f, 0.f, 0.f); }
  static __device__ float4 f32(type v) { return v; }
};

template <typename T>
struct Slice {
  using V = Vec4<T>;
  typename V::type va[kTasks], vb[kTasks];
  const T* row[kTasks];
  __device__ void init(const Args& a, int g, int tok0) {
#pragma unroll
    for (int u = 0; u < kTasks; ++u) {
      const int r = (g + kGroupThreads * u) / kQuads;
      if (r < kTokens) {
        const int t = tok0 + r;
        row[u] = t < a.T ? reinterpret_cast<const T*>(a.x) + (size_t)t * a.d : nullptr;
      } else {
        row[u] = wrow<T>(a, r - kTokens);
      }
    }
  }
  // ka / kb: the slice's first k in chunk A / B; la / lb: k past the end of each chunk
  __device__ void fetch(int g, int ka, int la, int kb, int lb) {
    const int kq = 4 * (g % kQuads);
#pragma unroll
    for (int u = 0; u < kTasks; ++u) {
      const T* r = row[u];
      va[u] = (r && ka + kq < la) ? *reinterpret_cast<const typename V::type*>(r + ka + kq) : V::zero();
      vb[u] = (r && kb + kq < lb) ? *reinterpret_cast<const typename V::type*>(r + kb + kq) : V::zero();
    }
  }
  __device__ void store(float* st, int g) const {
#pragma unroll
    for (int u = 0; u < kTasks; ++u) {
      const int r = (g + kGroupThreads * u) / kQuads;  // x rows then W rows: one pitch
      float* dst = st + r * kXP + 8 * (g % kQuads);
      const float4 A = V::f32(va[u]), B = V::f32(vb[u]);
      st4(dst, A.x, B.x, A.y, B.y);
      st4(dst + 4, A.z, B.z, A.w, B.w);
    }
  }
};
static_assert(kXP == kWP, "one pitch for the x and W rows of a slice");

// Two k of the slice for both chunks of the pair: 4 tokens x 4 rows of packed pairs.
__device__ __forceinline__ void mma_k2(float2 (&acc)[4][4], const float* xb, const float* wb, int kk) {
  float4 xv[4], wv[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) xv[i] = *reinterpret_cast<const float4*>(xb + 8 * i * kXP + 4 * kk);
#pragma unroll
  for (int j = 0; j < 4; ++j) wv[j] = *reinterpret_cast<const float4*>(wb + 16 * j * kWP + 4 * kk);
  // first k of the two for all 16 pairs, then the second: dependent updates sit 16 apart
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j)
      acc[i][j] = __ffma2_rn(make_float2(xv[i].x, xv[i].y), make_float2(wv[j].x, wv[j].y), acc[i][j]);
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j)
      acc[i][j] = __ffma2_rn(make_float2(xv[i].z, xv[i].w), make_float2(wv[j].z, wv[j].w), acc[i][j]);
}


template <typename T>
__global__ void __launch_bounds__(kThreads, 1) router_kernel(Args a) {
  extern __shared__ __align__(16) float smem[];
  __shared__ float lg_s[kTokens * kLP];
  __shared__ int ids_s[kTokens][DSCA_MAX_TOPK];
  __shared__ uint32_t emask[kRows];
  __shared__ int run_s[kRows];
  __shared__ int seg_s[kThreads / kRows][kRows];
  __shared__ int is_last;

  const int tid = threadIdx.x;
  const int q = tid / kGroupThreads;  // chunk group
  const int g = tid % kGroupThreads;
  const int tok0 = blockIdx.x * kTokens;
  const bool tau_bf16 = sizeof(T) == 2;
  if (tid < kRows) emask[tid] = 0u;

  if (a.logits_in != nullptr) {
    // logits from the tensor-core pass (router_tc.cu)
    for (int idx = tid; idx < kTokens * kRows; idx += kThreads) {
      const int t = idx / kRows, r = idx % kRows;
      lg_s[t * kLP + r] = (tok0 + t < a.T) ? a.logits_in[(size_t)(tok0 + t) * kRows + r] : 0.0f;
    }
    __syncthreads();
  } else {
  // ---------------- chunk partial sums, two chunks per group
  const int C = 32 * ((a.d + 255) / 256);
  const int nq = (a.d + C - 1) / C;
  const int qa = 2 * q, qb = 2 * q + 1;
  const int ka0 = qa * C, la = min(a.d, ka0 + C);
  const int kb0 = qb * C, lb = min(a.d, kb0 + C);  // lb <= kb0: no chunk B
  // warp w of the group, lane l, quad u = l / 4: tq = 4 (w & 1) + 2 (u & 1) + (l & 1),
  // rq = 8 (w >> 1) + 2 (u >> 1) + ((l >> 1) & 1)
  const int lq = g & 31, u4 = lq >> 2, wg = g >> 5;
  const int tq = ((wg & 1) << 2) | ((u4 & 1) << 1) | (lq & 1);
  const int rq = ((wg >> 1) << 3) | ((u4 >> 1) << 1) | ((lq >> 1) & 1);
  float2 acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = make_float2(0.0f, 0.0f);

  float* stage0 = smem + q * 2 * kStageFloats;
  if (qa < nq) {
    Slice<T> sl;
    sl.init(a, g, tok0);
    sl.fetch(g, ka0, la, kb0, lb);
    sl.store(stage0, g);
    group_sync(q);
    int s = 0;
    for (int o = 0; ka0 + o < la; o += kKS, s ^= 1) {
      const bool more = ka0 + o + kKS < la;
      if (more) sl.fetch(g, ka0 + o + kKS, la, kb0 + o + kKS, lb);  // in flight during the compute
      const float* st = stage0 + s * kStageFloats;
      const float* xb = st + tq * kXP;
      const float* wb = st + (kTokens + rq) * kWP;
      const int kmax = min(kKS, la - ka0 - o);  // a multiple of 8 (bf16) or 4 (fp32)
      if (kmax == kKS) {
#pragma unroll
        for (int kk = 0; kk < kKS / 2; ++kk) mma_k2(acc, xb, wb, kk);
      } else {
        for (int kk = 0; kk < kmax / 2; ++kk) mma_k2(acc, xb, wb, kk);
      }
      if (more) sl.store(stage0 + (s ^ 1) * kStageFloats, g);  // last read two slices ago
      group_sync(q);
    }
  }
  __syncthreads();  // staging buffers are reused for the partials below
  float* part = smem;  // [chunk][32 tokens][64 rows]
  if (qa < nq) {
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int t = tq + 8 * i, r = rq + 16 * j;
        part[(qa * kTokens + t) * kRows + r] = acc[i][j].x;
        if (qb < nq) part[(qb * kTokens + t) * kRows + r] = acc[i][j].y;
      }
  }
  __syncthreads();
  for (int idx = tid; idx < kTokens * kRows; idx += kThreads) {
    const int t = idx / kRows, r = idx % kRows;
    float tot = part[t * kRows + r];
    for (int qq = 1; qq < nq; ++qq) tot = __fadd_rn(tot, part[(qq * kTokens + t) * kRows + r]);
    lg_s[t * kLP + r] = tau_bf16 ? round_bf16(tot) : tot;
  }
  __syncthreads();
  }  // logits computed here

  select_block<T>(a, lg_s, ids_s, emask, run_s, seg_s, &is_last, (int)blockIdx.x, (int)gridDim.x, (int)gridDim.x);
}

}  // namespace router

int launch_router(const dsca_router_args* p, cudaStream_t stream, const float* logits_in) {
  static PerDeviceOnce attr_once[2];
  router::Args a;
  router::fill_args(p, &a);
  a.logits_in = logits_in;
  const int nblocks = (p->T + router::kTokens - 1) / router::kTokens;
  cudaError_t e = cudaSuccess;
  if (p->dtype == DSCA_BF16) {
    e = attr_once[0].run([] {
      return cudaFuncSetAttribute(router::router_kernel<__nv_bfloat16>,
                                  cudaFuncAttributeMaxDynamicSharedMemorySize, (int)router::kSmemBytes);
    });
    if (e == cudaSuccess)
      router::router_kernel<__nv_bfloat16><<<nblocks, router::kThreads, router::kSmemBytes, stream>>>(a);
  } else {
    e = attr_once[1].run([] {
      return cudaFuncSetAttribute(router::router_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  (int)router::kSmemBytes);
    });
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
