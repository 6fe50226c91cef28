// QoS planner scores — QoSPlanner.compute_token_scores and aggregate_expert_priority
// (src/qosmoe/planner.py:63-170) on the device.  They change no result: the expert-cache path
// orders its experts (and picks which ones to load) by these priorities.
//
//   count kernel:  n(e) = how many of the T tokens chose e first (one CTA).
//   token kernel:  one warp per token, 16-byte loads.  gain = |x - x_prev| (|x| without x_prev),
//                  attention factor = population variance of the token's logits row, penalty =
//                  target / (n(e0) + eps) with e0 the token's first choice, score =
//                  P (1 + gain (1 + attn) / (alpha d + beta rem + delta penalty)), -1e9 where
//                  the token is not valid.
//   expert kernel: one CTA per expert sums the scores of its (token, slot) assignments; each
//                  thread walks a fixed stride of assignments in order and the block reduces in
//                  a fixed tree, so the result does not depend on scheduling.
#include "common.cuh"

namespace dsca {
namespace qos {

constexpr int kWarps = 8;
constexpr int kMaxE = 4 * DSCA_MAX_EXPERTS;

template <typename T>
__device__ __forceinline__ float ld(const void* p, size_t i) {
  return static_cast<float>(reinterpret_cast<const T*>(p)[i]);
}
template <>
__device__ __forceinline__ float ld<__nv_bfloat16>(const void* p, size_t i) {
  return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
}

// 16 bytes of T as floats
template <typename T>
struct V16;
template <>
struct V16<__nv_bfloat16> {
  static constexpr int n = 8;
  static __device__ __forceinline__ void get(uint4 u, float* f) {
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      f[2 * i] = __uint_as_float(w[i] << 16);
      f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
    }
  }
};
template <>
struct V16<float> {
  static constexpr int n = 4;
  static __device__ __forceinline__ void get(uint4 u, float* f) {
    f[0] = __uint_as_float(u.x);
    f[1] = __uint_as_float(u.y);
    f[2] = __uint_as_float(u.z);
    f[3] = __uint_as_float(u.w);
  }
};

// first-choice counts n(e) over all T tokens (one CTA; into first_count [E])
__global__ void __launch_bounds__(1024) count_kernel(dsca_qos_args a, int32_t* first_count) {
  __shared__ int cnt[kMaxE];
  for (int e = threadIdx.x; e < a.E; e += blockDim.x) cnt[e] = 0;
  __syncthreads();
  for (int t = threadIdx.x; t < a.T; t += blockDim.x) {
    const int e = a.topk_ids[(size_t)t * a.top_k];
    if (e >= 0 && e < a.E) atomicAdd(&cnt[e], 1);
  }
  __syncthreads();
  for (int e = threadIdx.x; e < a.E; e += blockDim.x) first_count[e] = cnt[e];
}

// One warp scores token t (every lane returns the score; lane 0 stores it).  The row sums run in
// a fixed order: lane l takes the 16-byte vectors l, l + 32, ... of the row (all loads issued
// before the arithmetic), each vector's elements in index order into the lane's partial, then
// the xor butterfly.
template <typename T>
__device__ __forceinline__ float score_token(const dsca_qos_args& a, int t, const int32_t* first_count, int lane) {
  const size_t row = (size_t)t * a.d;
  float ss = 0.0f;
  constexpr int kE = V16<T>::n;
  const bool aligned = ((reinterpret_cast<uintptr_t>(a.x) | reinterpret_cast<uintptr_t>(a.x_prev)) & 15u) == 0;
  if ((a.d % kE) == 0 && aligned) {
    const uint4* xv = reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(a.x) + row);
    const uint4* pv = a.x_prev != nullptr ? reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(a.x_prev) + row)
                                          : nullptr;
    const int nv = a.d / kE;
    constexpr int kU = 8;
    for (int v0 = lane; v0 < nv; v0 += 32 * kU) {
      uint4 xu[kU], pu[kU];
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        const int v = v0 + 32 * u;
        xu[u] = v < nv ? xv[v] : make_uint4(0u, 0u, 0u, 0u);
        pu[u] = (pv != nullptr && v < nv) ? pv[v] : make_uint4(0u, 0u, 0u, 0u);
      }
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        if (v0 + 32 * u >= nv) break;
        float xf[kE], pf[kE];
        V16<T>::get(xu[u], xf);
        V16<T>::get(pu[u], pf);
#pragma unroll
        for (int i = 0; i < kE; ++i) {
          const float v = pv != nullptr ? __fsub_rn(xf[i], pf[i]) : xf[i];
          ss = __fmaf_rn(v, v, ss);
        }
      }
    }
  } else {
    for (int c = lane; c < a.d; c += 32) {
      float v = ld<T>(a.x, row + c);
      if (a.x_prev != nullptr) v = __fsub_rn(v, ld<T>(a.x_prev, row + c));
      ss = __fmaf_rn(v, v, ss);
    }
  }
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, off));
  const float gain = sqrtf(ss);
  // attention factor: population variance of the logits row (two passes)
  float attn = 0.0f;
  if (a.attention_mode == 0) {
    const size_t lrow = (size_t)t * a.E;
    float s = 0.0f;
    for (int e = lane; e < a.E; e += 32) s = __fadd_rn(s, ld<T>(a.logits, lrow + e));
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, off));
    const float mean = __fdiv_rn(s, (float)a.E);
    float q = 0.0f;
    for (int e = lane; e < a.E; e += 32) {
      const float dv = __fsub_rn(ld<T>(a.logits, lrow + e), mean);
      q = __fmaf_rn(dv, dv, q);
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) q = __fadd_rn(q, __shfl_xor_sync(0xffffffffu, q, off));
    attn = __fdiv_rn(q, (float)a.E);
  }
  float score = -1e9f;
  if (lane == 0) {
    const int e0 = a.topk_ids[(size_t)t * a.top_k];
    if (e0 < 0 || e0 >= a.E) {
      record_error(a.err, kErrIndex);
    } else {
      const float valid = a.valid != nullptr ? a.valid[t] : 1.0f;
      if (valid != 0.0f) {
        const float pri = a.seq_priority != nullptr ? a.seq_priority[t] : 1.0f;
        const float rem = a.remaining != nullptr ? a.remaining[t] : 0.0f;
        const float penalty = __fdiv_rn(a.target_batch, __fadd_rn((float)first_count[e0], a.epsilon));
        const float denom = __fadd_rn(__fadd_rn(__fmul_rn(a.alpha, (float)a.d), __fmul_rn(a.beta, rem)),
                                      __fmul_rn(a.delta, penalty));
        const float value = __fdiv_rn(__fmul_rn(gain, __fadd_rn(1.0f, attn)), denom);
        score = __fmul_rn(pri, __fadd_rn(1.0f, value));
      }
    }
    a.token_score[t] = score;
  }
  return __shfl_sync(0xffffffffu, score, 0);
}

// One warp per token.
template <typename T>
__global__ void __launch_bounds__(kWarps * 32) token_kernel(dsca_qos_args a, const int32_t* first_count) {
  const int t = (int)(blockIdx.x * kWarps + (threadIdx.x >> 5));
  if (t >= a.T) return;
  score_token<T>(a, t, first_count, (int)(threadIdx.x & 31));
}

// The one-kernel form: CTA b scores tokens [32 b, 32 b + 32) (one warp per token), sums the scores
// of its own (token, slot) assignments per expert in token-then-slot order into partial[b], and
// the last CTA to finish adds the partials in CTA order (four runs of CTAs, eight loads in flight
// each, then the four run sums in order).  first_count is read by every CTA before it arrives;
// the last CTA zeroes it (when the router accumulated it) and the done counter.
constexpr int kFusedTokens = 32;
template <typename T>
__global__ void __launch_bounds__(kWarps * 32) fused_kernel(dsca_qos_args a, const int32_t* first_count,
                                                            int zero_first_count) {
  __shared__ float sc[kFusedTokens];
  __shared__ int ids_s[kFusedTokens * DSCA_MAX_TOPK];
  __shared__ float run[4][kMaxE];
  __shared__ int is_last;
  const int warp = (int)(threadIdx.x >> 5), lane = (int)(threadIdx.x & 31), tid = (int)threadIdx.x;
  const int t0 = (int)blockIdx.x * kFusedTokens, k = a.top_k, E = a.E;
  for (int tl = warp; tl < kFusedTokens; tl += kWarps) {
    const int t = t0 + tl;
    const float s = t < a.T ? score_token<T>(a, t, first_count, lane) : 0.0f;
    if (lane == 0) sc[tl] = s;
  }
  for (int i = tid; i < kFusedTokens * k; i += kWarps * 32) {
    const int t = t0 + i / k;
    ids_s[i] = t < a.T ? a.topk_ids[(size_t)t0 * k + i] : -1;
  }
  __syncthreads();
  for (int e = tid; e < E; e += kWarps * 32) {
    float p = 0.0f;
    for (int i = 0; i < kFusedTokens * k; ++i)
      if (ids_s[i] == e) p = __fadd_rn(p, sc[i / k]);
    a.partial[(size_t)blockIdx.x * E + e] = p;
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    const uint32_t prev = atomicAdd(a.done_counter, 1u);
    is_last = prev == gridDim.x - 1u;
    __threadfence();
  }
  __syncthreads();
  if (!is_last) return;
  const int nb = (int)gridDim.x, per = (nb + 3) / 4;
  for (int idx = tid; idx < 4 * E; idx += kWarps * 32) {
    const int e = idx % E, c = idx / E;
    const int b0 = min(nb, c * per), b1 = min(nb, b0 + per);
    float p = 0.0f;
    for (int b = b0; b < b1; b += 8) {
      float v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) v[u] = b + u < b1 ? __ldcg(a.partial + (size_t)(b + u) * E + e) : 0.0f;
#pragma unroll
      for (int u = 0; u < 8; ++u)
        if (b + u < b1) p = __fadd_rn(p, v[u]);
    }
    run[c][e] = p;
  }
  __syncthreads();
  for (int e = tid; e < E; e += kWarps * 32) {
    a.expert_priority[e] = __fadd_rn(__fadd_rn(__fadd_rn(run[0][e], run[1][e]), run[2][e]), run[3][e]);
    if (zero_first_count) a.first_counts[e] = 0;
  }
  if (tid == 0) *a.done_counter = 0u;
}

// One CTA per expert sums the scores of its (token, slot) assignments; each thread walks a fixed
// stride of the assignments in order and the block reduces in a fixed tree, so the result does
// not depend on scheduling.  Eight loads in flight per thread.
__global__ void __launch_bounds__(256) expert_kernel(dsca_qos_args a) {
  __shared__ float part[256];
  const int e = blockIdx.x, tid = threadIdx.x;
  const int n = a.T * a.top_k;
  float s = 0.0f;
  constexpr int kU = 8;
  for (int w0 = tid; w0 < n; w0 += 256 * kU) {
    int ids[kU];
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const int w = w0 + 256 * u;
      ids[u] = w < n ? a.topk_ids[w] : -1;
    }
#pragma unroll
    for (int u = 0; u < kU; ++u)
      if (ids[u] == e) s = __fadd_rn(s, a.token_score[(w0 + 256 * u) / a.top_k]);
  }
  part[tid] = s;
  __syncthreads();
  for (int h = 128; h >= 1; h >>= 1) {
    if (tid < h) part[tid] = __fadd_rn(part[tid], part[tid + h]);
    __syncthreads();
  }
  if (tid == 0) a.expert_priority[e] = part[0];
}

}  // namespace qos

int launch_qos(const dsca_qos_args* a, cudaStream_t stream) {
  // the first-choice counts: from the router (first_counts), else counted here into the
  // expert_priority array (E floats long, overwritten with the priorities once every token has
  // read the counts)
  const bool from_router = a->first_counts != nullptr;
  int32_t* first_count = from_router ? a->first_counts : reinterpret_cast<int32_t*>(a->expert_priority);
  if (!from_router) qos::count_kernel<<<1, 1024, 0, stream>>>(*a, first_count);
  if (a->partial != nullptr && a->done_counter != nullptr) {
    const int blocks = (a->T + qos::kFusedTokens - 1) / qos::kFusedTokens;
    if (blocks > 0) {
      if (a->dtype == DSCA_BF16)
        qos::fused_kernel<__nv_bfloat16><<<blocks, qos::kWarps * 32, 0, stream>>>(*a, first_count, from_router);
      else
        qos::fused_kernel<float><<<blocks, qos::kWarps * 32, 0, stream>>>(*a, first_count, from_router);
    }
    return cudaGetLastError() == cudaSuccess ? DSCA_OK : DSCA_ERR_CUDA;
  }
  const int blocks = (a->T + qos::kWarps - 1) / qos::kWarps;
  if (blocks > 0) {
    if (a->dtype == DSCA_BF16)
      qos::token_kernel<__nv_bfloat16><<<blocks, qos::kWarps * 32, 0, stream>>>(*a, first_count);
    else
      qos::token_kernel<float><<<blocks, qos::kWarps * 32, 0, stream>>>(*a, first_count);
  }
  qos::expert_kernel<<<a->E, 256, 0, stream>>>(*a);
  return cudaGetLastError() == cudaSuccess ? DSCA_OK : DSCA_ERR_CUDA;
}

}  // namespace dsca
