// QoS planner scores — QoSPlanner.compute_token_scores and aggregate_expert_priority
// (src/qosmoe/planner.py:63-170) on the device.  They change no result: the expert-cache path
// orders its experts (and picks which ones to load) by these priorities.
//
//   token kernel:  one warp per token.  gain = |x - x_prev| (|x| without x_prev), attention
//                  factor = population variance of the token's logits row, penalty = target /
//                  (n(e0) + eps) with e0 the token's first choice and n the first-choice count
//                  over all T tokens (each CTA counts them into shared memory), score =
//                  P (1 + gain (1 + attn) / (alpha d + beta rem + delta penalty)), -1e9 where
//                  the token is not valid.
//   expert kernel: one CTA per expert sums the scores of its (token, slot) assignments; each
//                  thread walks a fixed stride of assignments in order and the block reduces in
//                  a fixed tree, so the result does not depend on scheduling.
#include "common.cuh"

namespace dsca {
namespace qos {

constexpr int kWarps = 8;
constexpr int kTokensPerWarp = 8;
constexpr int kMaxE = 4 * DSCA_MAX_EXPERTS;

template <typename T>
__device__ __forceinline__ float ld(const void* p, size_t i) {
  return static_cast<float>(reinterpret_cast<const T*>(p)[i]);
}
template <>
__device__ __forceinline__ float ld<__nv_bfloat16>(const void* p, size_t i) {
  return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
}

template <typename T>
__global__ void __launch_bounds__(kWarps * 32) token_kernel(dsca_qos_args a) {
  __shared__ int first_count[kMaxE];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  for (int e = tid; e < a.E; e += blockDim.x) first_count[e] = 0;
  __syncthreads();
  for (int t = tid; t < a.T; t += blockDim.x) {
    const int e = a.topk_ids[(size_t)t * a.top_k];
    if (e >= 0 && e < a.E) atomicAdd(&first_count[e], 1);
  }
  __syncthreads();
  const float hidden_cost = (float)a.d;
  for (int i = 0; i < kTokensPerWarp; ++i) {
    const int t = (blockIdx.x * kWarps + warp) * kTokensPerWarp + i;
    if (t >= a.T) break;
    // information gain: |x - x_prev| over the row, lane partials in index order, then the
    // xor butterfly
    float ss = 0.0f;
    const size_t row = (size_t)t * a.d;
    for (int c = lane; c < a.d; c += 32) {
      float v = ld<T>(a.x, row + c);
      if (a.x_prev != nullptr) v = __fsub_rn(v, ld<T>(a.x_prev, row + c));
      ss = __fmaf_rn(v, v, ss);
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
    if (lane == 0) {
      const int e0 = a.topk_ids[(size_t)t * a.top_k];
      float score = -1e9f;
      if (e0 < 0 || e0 >= a.E) {
        record_error(a.err, kErrIndex);
      } else {
        const float valid = a.valid != nullptr ? a.valid[t] : 1.0f;
        if (valid != 0.0f) {
          const float pri = a.seq_priority != nullptr ? a.seq_priority[t] : 1.0f;
          const float rem = a.remaining != nullptr ? a.remaining[t] : 0.0f;
          const float penalty = __fdiv_rn(a.target_batch, __fadd_rn((float)first_count[e0], a.epsilon));
          const float denom = __fadd_rn(__fadd_rn(__fmul_rn(a.alpha, hidden_cost), __fmul_rn(a.beta, rem)),
                                        __fmul_rn(a.delta, penalty));
          const float value = __fdiv_rn(__fmul_rn(gain, __fadd_rn(1.0f, attn)), denom);
          score = __fmul_rn(pri, __fadd_rn(1.0f, value));
        }
      }
      a.token_score[t] = score;
    }
  }
}

__global__ void __launch_bounds__(256) expert_kernel(dsca_qos_args a) {
  __shared__ float part[256];
  const int e = blockIdx.x, tid = threadIdx.x;
  const int n = a.T * a.top_k;
  float s = 0.0f;
  for (int w = tid; w < n; w += 256)
    if (a.topk_ids[w] == e) s = __fadd_rn(s, a.token_score[w / a.top_k]);
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
  constexpr int per_block = qos::kWarps * qos::kTokensPerWarp;
  const int blocks = (a->T + per_block - 1) / per_block;
  if (blocks > 0) {
    if (a->dtype == DSCA_BF16)
      qos::token_kernel<__nv_bfloat16><<<blocks, qos::kWarps * 32, 0, stream>>>(*a);
    else
      qos::token_kernel<float><<<blocks, qos::kWarps * 32, 0, stream>>>(*a);
  }
  qos::expert_kernel<<<a->E, 256, 0, stream>>>(*a);
  return cudaGetLastError() == cudaSuccess ? DSCA_OK : DSCA_ERR_CUDA;
}

}  // namespace dsca
