// K1 — router: logits, softmax, top-1 / top-k, shared-expert gate, per-block histogram and
// in-block stable ranks, fused in one launch.
//
// Reference semantics: Router.standard_forward (src/harmonymoe/router.py:52-63) and the
// argmax at src/qosmoe/moe_layer.py:287 for the Switch top-1 block; gate / softmax(fp32) /
// topk / renorm / cast of ShardedQwenMoE.forward (qwen_ep_adapter/qwen_ep.py:48-53) and the
// shared-expert gate sigmoid (qwen_ep.py:94) for the Qwen block.
//
// Layout: one CTA = 8 warps = 32 tokens (DSCA_ROUTER_TOKENS).  Warp w owns tokens 4w..4w+3;
// lane L owns router rows L and L+32 (E + shared gate <= 64).  x and W stream through shared
// memory in 64-wide slices of d (converted to fp32, W rows padded to 68 floats so the float4
// reads of 8 consecutive lanes hit distinct banks); the next slice is fetched into registers
// while the current one is consumed.  Each logit is one thread's sequential fma chain over
// i = 0..d-1, so the value is fixed by the data alone.  Softmax and selection then run inside
// the warp that already holds the token's logits (no shared-memory round trip).
#include "common.cuh"

namespace dsca {
namespace router {

constexpr int kTokens = DSCA_ROUTER_TOKENS;  // 32
constexpr int kThreads = 256;
constexpr int kRows = 64;                   // router rows per CTA (E experts + shared gate)
constexpr int kDK = 64;                     // d slice
constexpr int kXPitch = kDK + 4;
constexpr int kWPitch = kDK + 4;

template <typename T>
struct Loader;

template <>
struct Loader<__nv_bfloat16> {
  // x slice: 32 tokens x 64 values = 256 x 8 bf16 (one uint4 per thread)
  // W slice: 64 rows x 64 values = 512 x 8 bf16 (two uint4 per thread)
  static constexpr int kXVec = 1, kWVec = 2;
  uint4 xr[kXVec], wr[kWVec];
  __device__ void fetch(const __nv_bfloat16* x, const __nv_bfloat16* W, int T, int d, int rows,
                        int tok0, int k0) {
    for (int v = 0; v < kXVec; ++v) {
      int idx = threadIdx.x + v * kThreads;  // 0..255
      int t = idx >> 3, c = (idx & 7) * 8;
      int tok = tok0 + t, col = k0 + c;
      xr[v] = make_uint4(0, 0, 0, 0);
      if (tok < T && col < d) xr[v] = *reinterpret_cast<const uint4*>(x + (size_t)tok * d + col);
    }
    for (int v = 0; v < kWVec; ++v) {
      int idx = threadIdx.x + v * kThreads;  // 0..511
      int r = idx >> 3, c = (idx & 7) * 8;
      int col = k0 + c;
      wr[v] = make_uint4(0, 0, 0, 0);
      if (r < rows && col < d) wr[v] = *reinterpret_cast<const uint4*>(W + (size_t)r * d + col);
    }
  }
  __device__ void store(float* xs, float* ws) {
    for (int v = 0; v < kXVec; ++v) {
      int idx = threadIdx.x + v * kThreads;
      int t = idx >> 3, c = (idx & 7) * 8;
      const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(&xr[v]);
      float4 a = make_float4(__bfloat162float(h[0]), __bfloat162float(h[1]), __bfloat162float(h[2]),
                             __bfloat162float(h[3]));
      float4 b = make_float4(__bfloat162float(h[4]), __bfloat162float(h[5]), __bfloat162float(h[6]),
                             __bfloat162float(h[7]));
      *reinterpret_cast<float4*>(xs + t * kXPitch + c) = a;
      *reinterpret_cast<float4*>(xs + t * kXPitch + c + 4) = b;
    }
    for (int v = 0; v < kWVec; ++v) {
      int idx = threadIdx.x + v * kThreads;
      int r = idx >> 3, c = (idx & 7) * 8;
      const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(&wr[v]);
      float4 a = make_float4(__bfloat162float(h[0]), __bfloat162float(h[1]), __bfloat162float(h[2]),
                             __bfloat162float(h[3]));
      float4 b = make_float4(__bfloat162float(h[4]), __bfloat162float(h[5]), __bfloat162float(h[6]),
                             __bfloat162float(h[7]));
      *reinterpret_cast<float4*>(ws + r * kWPitch + c) = a;
      *reinterpret_cast<float4*>(ws + r * kWPitch + c + 4) = b;
    }
  }
};

template <>
struct Loader<float> {
  // x slice: 32 x 64 floats = 512 float4 (two per thread); W: 64 x 64 = 1024 float4 (four)
  static constexpr int kXVec = 2, kWVec = 4;
  float4 xr[kXVec], wr[kWVec];
  __device__ void fetch(const float* x, const float* W, int T, int d, int rows, int tok0, int k0) {
    for (int v = 0; v < kXVec; ++v) {
      int idx = threadIdx.x + v * kThreads;  // 0..511
      int t = idx >> 4, c = (idx & 15) * 4;
      int tok = tok0 + t, col = k0 + c;
      xr[v] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (tok < T && col < d) xr[v] = *reinterpret_cast<const float4*>(x + (size_t)tok * d + col);
    }
    for (int v = 0; v < kWVec; ++v) {
      int idx = threadIdx.x + v * kThreads;  // 0..1023
      int r = idx >> 4, c = (idx & 15) * 4;
      int col = k0 + c;
      wr[v] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (r < rows && col < d) wr[v] = *reinterpret_cast<const float4*>(W + (size_t)r * d + col);
    }
  }
  __device__ void store(float* xs, float* ws) {
    for (int v = 0; v < kXVec; ++v) {
      int idx = threadIdx.x + v * kThreads;
      int t = idx >> 4, c = (idx & 15) * 4;
      *reinterpret_cast<float4*>(xs + t * kXPitch + c) = xr[v];
    }
    for (int v = 0; v < kWVec; ++v) {
      int idx = threadIdx.x + v * kThreads;
      int r = idx >> 4, c = (idx & 15) * 4;
      *reinterpret_cast<float4*>(ws + r * kWPitch + c) = wr[v];
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
};

template <typename T>
__global__ void __launch_bounds__(kThreads, 2) router_kernel(Args a) {
  __shared__ __align__(16) float xs[kTokens * kXPitch];
  __shared__ __align__(16) float ws[kRows * kWPitch];
  __shared__ int ids_s[kTokens][DSCA_MAX_TOPK];

  const int warp = warp_id(), lane = lane_id();
  const int tok0 = blockIdx.x * kTokens;
  const int E = a.E;
  const bool has_sg = a.w_shared_gate != nullptr;
  const T* x = reinterpret_cast<const T*>(a.x);
  const T* Wr = reinterpret_cast<const T*>(a.w_router);
  const T* Wg = reinterpret_cast<const T*>(a.w_shared_gate);

  // rows 0..E-1 = router, row E = shared gate.  Build a virtual [rows, d] view: the loader
  // reads row r < E from Wr and row E from Wg.
  float acc[4][2];
#pragma unroll
  for (int i = 0; i < 4; ++i) acc[i][0] = acc[i][1] = 0.0f;

  Loader<T> ld;
  auto fetch = [&](int k0) {
    ld.fetch(x, Wr, a.T, a.d, E, tok0, k0);
    if (has_sg) {
      // the shared-gate row replaces row E of the W slice (loader zero-filled it)
      constexpr int per_row = kDK / (16 / (int)sizeof(T));  // vectors per 64-wide row
      for (int v = 0; v < Loader<T>::kWVec; ++v) {
        int idx = threadIdx.x + v * kThreads;
        int r = idx / per_row, c = (idx % per_row) * (16 / (int)sizeof(T));
        if (r == E && k0 + c < a.d) {
          if constexpr (sizeof(T) == 2)
            ld.wr[v] = *reinterpret_cast<const uint4*>(Wg + k0 + c);
          else
            ld.wr[v] = *reinterpret_cast<const float4*>(Wg + k0 + c);
        }
      }
    }
  };

  const int nslices = (a.d + kDK - 1) / kDK;
  fetch(0);
  for (int s = 0; s < nslices; ++s) {
    __syncthreads();  // previous slice fully consumed
    ld.store(xs, ws);
    __syncthreads();
    if (s + 1 < nslices) fetch((s + 1) * kDK);
    const int kmax = min(kDK, a.d - s * kDK);
    const float* w0 = ws + lane * kWPitch;
    const float* w1 = ws + (lane + 32) * kWPitch;
    const float* xw = xs + (warp * 4) * kXPitch;
    int k = 0;
    for (; k + 4 <= kmax; k += 4) {
      float4 wa = *reinterpret_cast<const float4*>(w0 + k);
      float4 wb = *reinterpret_cast<const float4*>(w1 + k);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        float4 xv = *reinterpret_cast<const float4*>(xw + i * kXPitch + k);
        acc[i][0] = __fmaf_rn(xv.x, wa.x, acc[i][0]);
        acc[i][0] = __fmaf_rn(xv.y, wa.y, acc[i][0]);
        acc[i][0] = __fmaf_rn(xv.z, wa.z, acc[i][0]);
        acc[i][0] = __fmaf_rn(xv.w, wa.w, acc[i][0]);
        acc[i][1] = __fmaf_rn(xv.x, wb.x, acc[i][1]);
        acc[i][1] = __fmaf_rn(xv.y, wb.y, acc[i][1]);
        acc[i][1] = __fmaf_rn(xv.z, wb.z, acc[i][1]);
        acc[i][1] = __fmaf_rn(xv.w, wb.w, acc[i][1]);
      }
    }
    for (; k < kmax; ++k) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        acc[i][0] = __fmaf_rn(xw[i * kXPitch + k], w0[k], acc[i][0]);
        acc[i][1] = __fmaf_rn(xw[i * kXPitch + k], w1[k], acc[i][1]);
      }
    }
  }

  const bool tau_bf16 = sizeof(T) == 2;
  const int e0 = lane, e1 = lane + 32;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int tl = warp * 4 + i;
    const int t = tok0 + tl;
    float l0 = tau_bf16 ? round_bf16(acc[i][0]) : acc[i][0];
    float l1 = tau_bf16 ? round_bf16(acc[i][1]) : acc[i][1];
    const bool valid = t < a.T;
    if (valid) {
      if (e0 < E) store_logit<T>(a.logits, (size_t)t * E + e0, l0);
      if (e1 < E) store_logit<T>(a.logits, (size_t)t * E + e1, l1);
      if (has_sg && a.shared_gate != nullptr) {
        float z = (e0 == E) ? l0 : l1;
        if (e0 == E || e1 == E) a.shared_gate[t] = 1.0f / (1.0f + expf(-z));
      }
    }
    // softmax over the E router logits of this token
    float v0 = (e0 < E) ? l0 : -INFINITY;
    float v1 = (e1 < E) ? l1 : -INFINITY;
    float m = fmaxf(v0, v1);
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
    float x0 = (e0 < E) ? exp_neg(__fsub_rn(l0, m)) : 0.0f;
    float x1 = (e1 < E) ? exp_neg(__fsub_rn(l1, m)) : 0.0f;
    float part = (e0 < E) ? __fadd_rn(0.0f, x0) : 0.0f;
    if (e1 < E) part = __fadd_rn(part, x1);
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) part = __fadd_rn(part, __shfl_xor_sync(0xffffffffu, part, off));
    float p0 = (e0 < E) ? __fdiv_rn(x0, part) : -INFINITY;
    float p1 = (e1 < E) ? __fdiv_rn(x1, part) : -INFINITY;

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
        float ov = __shfl_xor_sync(0xffffffffu, bv, off);
        int oi = __shfl_xor_sync(0xffffffffu, bi, off);
        if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
      }
      if (lane == 0) {
        ids_s[tl][0] = valid ? bi : -1;
        if (valid) {
          a.topk_ids[t] = bi;
          a.topk_w[t] = (a.weight_round_bf16 && !tau_bf16) ? round_bf16(bv) : bv;
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
          float ov = __shfl_xor_sync(0xffffffffu, bv, off);
          int oi = __shfl_xor_sync(0xffffffffu, bi, off);
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

  // per-block histogram and stable in-block ranks (token order, slot order)
  const int k = (a.mode == DSCA_ROUTE_SWITCH_TOP1) ? 1 : a.top_k;
  for (int e = threadIdx.x; e < E; e += kThreads) {
    int c = 0;
    for (int tl = 0; tl < kTokens; ++tl)
      for (int j = 0; j < k; ++j) c += (ids_s[tl][j] == e);
    a.block_hist[(size_t)blockIdx.x * E + e] = c;
  }
  for (int idx = threadIdx.x; idx < kTokens * k; idx += kThreads) {
    int tl = idx / k, j = idx % k;
    int t = tok0 + tl;
    int e = ids_s[tl][j];
    if (t >= a.T || e < 0) continue;
    int r = 0;
    for (int u = 0; u < tl; ++u)
      for (int jj = 0; jj < k; ++jj) r += (ids_s[u][jj] == e);
    a.local_rank[(size_t)t * k + j] = r;
  }
}

}  // namespace router

int launch_router(const dsca_router_args* p, cudaStream_t stream) {
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
  const int nblocks = (p->T + router::kTokens - 1) / router::kTokens;
  if (p->dtype == DSCA_BF16)
    router::router_kernel<__nv_bfloat16><<<nblocks, router::kThreads, 0, stream>>>(a);
  else
    router::router_kernel<float><<<nblocks, router::kThreads, 0, stream>>>(a);
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
