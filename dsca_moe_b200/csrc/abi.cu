// extern "C" entry points: argument validation, then the kernel launches in router.cu,
// dispatch.cu, gemm_sm100.cu and gemm_simt.cu.  No entry point allocates device memory.
#include <stdio.h>

#include "common.cuh"

namespace dsca {
int launch_router(const dsca_router_args* p, cudaStream_t stream, const float* logits_in = nullptr);
int launch_router_tc(const dsca_router_args* a, cudaStream_t stream);
int launch_router_pack_i8(const void* rows, int R, int d, void* slices, int32_t* exps, cudaStream_t stream);
bool router_tc_fused_supported(int d);
int launch_exp_eval(const float* x, float* y, int n, cudaStream_t stream);
int launch_scan(const dsca_scan_args* a, cudaStream_t stream);
int launch_permute(const dsca_permute_args* a, cudaStream_t stream);
int launch_combine(const dsca_combine_args* a, cudaStream_t stream);
int launch_qos(const dsca_qos_args* a, cudaStream_t stream);
int launch_grouped_ffn_bf16(const dsca_ffn_args* f, int num_sms, cudaStream_t stream);
int launch_grouped_ffn_f32(const dsca_ffn_args* f, int num_sms, cudaStream_t stream);
int launch_grouped_ffn_fp8(const dsca_ffn_args* f, int num_sms, cudaStream_t stream);
int launch_grouped_ffn_fp8_tmem(const dsca_ffn_args* f, int num_sms, cudaStream_t stream);
int launch_grouped_ffn_f8_split(const dsca_ffn_args* f, int num_sms, cudaStream_t stream);
int launch_split_rows(const void* src, int ld, int rows, const int32_t* rows_dev, int K, void* dst, float* inv_scale,
                      cudaStream_t stream);
}  // namespace dsca

namespace {

struct DevInfo {
  int device = -1;
  int num_sms = 0;
  int major = 0;
};

// per-device cache of the SM count (queried once per device)
DevInfo g_dev[64];

int device_info(int* num_sms, int* major) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return DSCA_ERR_CUDA;
  DevInfo& d = g_dev[dev];
  if (d.device != dev) {
    cudaDeviceProp prop;
    if (cudaGetDeviceProperties(&prop, dev) != cudaSuccess) return DSCA_ERR_CUDA;
    d.num_sms = prop.multiProcessorCount;
    d.major = prop.major;
    d.device = dev;
  }
  *num_sms = d.num_sms;
  *major = d.major;
  return DSCA_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

extern "C" {

const char* dsca_version(void) { return "dsca_b200 0.1 (sm_100a)"; }

const char* dsca_status_string(int s) {
  switch (s) {
    case DSCA_OK: return "ok";
    case DSCA_ERR_BAD_ARG: return "bad argument";
    case DSCA_ERR_CAPACITY: return "capacity exceeded";
    case DSCA_ERR_WAIT_TIMEOUT: return "device wait timed out";
    case DSCA_ERR_CUDA: return "CUDA error";
    case DSCA_ERR_DEVICE_INDEX: return "device bounds check failed";
    case DSCA_ERR_UNSUPPORTED: return "unsupported device (needs sm_100)";
    default: return "unknown status";
  }
}

int dsca_device_info(int* num_sms, int* is_sm100) {
  if (num_sms == nullptr || is_sm100 == nullptr) return DSCA_ERR_BAD_ARG;
  int major = 0;
  int rc = device_info(num_sms, &major);
  if (rc) return rc;
  *is_sm100 = major == 10 ? 1 : 0;
  return DSCA_OK;
}

int dsca_router_topk(const dsca_router_args* a, dsca_stream_t stream) {
  if (a == nullptr || a->x == nullptr || a->w_router == nullptr || a->logits == nullptr ||
      a->topk_ids == nullptr || a->topk_w == nullptr || a->block_hist == nullptr ||
      a->local_rank == nullptr)
    return DSCA_ERR_BAD_ARG;
  if (a->T < 0 || a->d <= 0 || a->E <= 0) return DSCA_ERR_BAD_ARG;
  if (a->dtype != DSCA_BF16 && a->dtype != DSCA_F32) return DSCA_ERR_BAD_ARG;
  if (a->mode != DSCA_ROUTE_SWITCH_TOP1 && a->mode != DSCA_ROUTE_SOFTMAX_TOPK) return DSCA_ERR_BAD_ARG;
  const int k = a->mode == DSCA_ROUTE_SWITCH_TOP1 ? 1 : a->top_k;
  if (k <= 0 || k > DSCA_MAX_TOPK || k > a->E) return DSCA_ERR_BAD_ARG;
  if (a->E + (a->w_shared_gate ? 1 : 0) > DSCA_MAX_EXPERTS) return DSCA_ERR_CAPACITY;
  // 16-byte vector loads of x / W rows
  const int vec = a->dtype == DSCA_BF16 ? 8 : 4;
  if (a->d % vec != 0 || !aligned16(a->x) || !aligned16(a->w_router) ||
      (a->w_shared_gate && !aligned16(a->w_shared_gate)))
    return DSCA_ERR_BAD_ARG;
  // the fused scan takes all four outputs or none
  const int nscan = (a->counts != nullptr) + (a->offsets != nullptr) + (a->block_base != nullptr) +
                    (a->done_counter != nullptr);
  if (nscan != 0 && nscan != 4) return DSCA_ERR_BAD_ARG;
  // the tensor-core logits: w_slices and w_exp, bf16 only; the scratch buffers (all three) only
  // for d > 2048
  const bool tc = a->w_slices != nullptr || a->w_exp != nullptr;
  if (tc) {
    if (a->w_slices == nullptr || a->w_exp == nullptr || a->dtype != DSCA_BF16 || !aligned16(a->w_slices) ||
        a->d > 32768)
      return DSCA_ERR_BAD_ARG;
    if (!dsca::router_tc_fused_supported(a->d) &&
        (a->x_slices == nullptr || a->x_exp == nullptr || a->logits_f32 == nullptr || !aligned16(a->x_slices) ||
         !aligned16(a->logits_f32)))
      return DSCA_ERR_BAD_ARG;
  }
  if (a->T == 0) return DSCA_OK;
  if (tc) return dsca::launch_router_tc(a, reinterpret_cast<cudaStream_t>(stream));
  return dsca::launch_router(a, reinterpret_cast<cudaStream_t>(stream));
}

int dsca_router_pack_i8(const void* rows, int R, int d, void* w_slices, int32_t* w_exp, dsca_stream_t stream) {
  if (rows == nullptr || w_slices == nullptr || w_exp == nullptr || R <= 0 || R > DSCA_MAX_EXPERTS || d <= 0 ||
      d % 8 != 0 || d > 32768 || !aligned16(rows) || !aligned16(w_slices))
    return DSCA_ERR_BAD_ARG;
  return dsca::launch_router_pack_i8(rows, R, d, w_slices, w_exp, reinterpret_cast<cudaStream_t>(stream));
}

int dsca_dispatch_scan(const dsca_scan_args* a, dsca_stream_t stream) {
  if (a == nullptr || a->block_hist == nullptr || a->counts == nullptr || a->offsets == nullptr ||
      a->block_base == nullptr || a->nblocks < 0 || a->E <= 0)
    return DSCA_ERR_BAD_ARG;
  if (a->E > 4 * DSCA_MAX_EXPERTS) return DSCA_ERR_CAPACITY;
  return dsca::launch_scan(a, reinterpret_cast<cudaStream_t>(stream));
}

int dsca_permute(const dsca_permute_args* a, dsca_stream_t stream) {
  if (a == nullptr || a->x == nullptr || a->topk_ids == nullptr || a->local_rank == nullptr ||
      a->block_base == nullptr || a->out == nullptr || a->token_row == nullptr || a->T < 0 ||
      a->d <= 0 || a->E <= 0 || a->top_k <= 0 || a->top_k > DSCA_MAX_TOPK || a->capacity < 0)
    return DSCA_ERR_BAD_ARG;
  if (a->dtype != DSCA_BF16 && a->dtype != DSCA_F32) return DSCA_ERR_BAD_ARG;
  const int esz = a->dtype == DSCA_BF16 ? 2 : 4;
  if (((size_t)a->d * esz) % 16 != 0 || !aligned16(a->x) || !aligned16(a->out)) return DSCA_ERR_BAD_ARG;
  if (a->cum_split == nullptr) {
    if (a->offsets == nullptr) return DSCA_ERR_BAD_ARG;
  } else {
    if (a->dest_base == nullptr || a->G <= 0 || a->G > DSCA_MAX_GPUS) return DSCA_ERR_BAD_ARG;
  }
  if (a->out_e4m3) {
    if (a->dtype != DSCA_BF16 || a->out_f16 || a->out_scale == nullptr || a->d % 8 != 0) return DSCA_ERR_BAD_ARG;
    if (a->x_q != nullptr && (a->x_scale == nullptr || !aligned16(a->x_q))) return DSCA_ERR_BAD_ARG;
  }
  return dsca::launch_permute(a, reinterpret_cast<cudaStream_t>(stream));
}

int dsca_split_rows(const dsca_split_args* a, dsca_stream_t stream) {
  if (a == nullptr || a->rows < 0 || a->K <= 0 || a->K % 8 != 0 || a->ld < a->K || a->ld % 8 != 0) return DSCA_ERR_BAD_ARG;
  if (a->rows == 0) return DSCA_OK;
  if (a->src == nullptr || a->dst == nullptr || a->inv_scale == nullptr || !aligned16(a->src) || !aligned16(a->dst))
    return DSCA_ERR_BAD_ARG;
  return dsca::launch_split_rows(a->src, a->ld, a->rows, a->rows_dev, a->K, a->dst, a->inv_scale,
                                 reinterpret_cast<cudaStream_t>(stream));
}

int dsca_grouped_ffn(const dsca_ffn_args* f, dsca_stream_t stream) {
  if (f != nullptr && f->shared_handoff != 0 && f->shared_handoff != 1) return DSCA_ERR_BAD_ARG;
  if (f == nullptr || f->a == nullptr || f->w1 == nullptr || f->w2 == nullptr || f->h == nullptr ||
      f->y == nullptr || f->group_offsets == nullptr)
    return DSCA_ERR_BAD_ARG;
  if (f->num_groups <= 0 || f->num_groups > 256 || f->capacity < 0 || f->d <= 0 || f->num_experts_w <= 0)
    return f->num_groups > 256 ? DSCA_ERR_CAPACITY : DSCA_ERR_BAD_ARG;
  if (f->act != DSCA_ACT_RELU && f->act != DSCA_ACT_SWIGLU) return DSCA_ERR_BAD_ARG;
  const bool glu = f->act == DSCA_ACT_SWIGLU;
  // packing contract (see dsca_b200.h)
  if (f->n1p <= 0 || f->n1p % 256 != 0 || f->dp < f->d || f->dp % 256 != 0) return DSCA_ERR_BAD_ARG;
  if (f->ip != (glu ? f->n1p / 2 : f->n1p)) return DSCA_ERR_BAD_ARG;
  if (f->d % 8 != 0) return DSCA_ERR_BAD_ARG;
  if (f->shared_rows > 0) {
    if (f->xs == nullptr || f->ws1 == nullptr || f->ws2 == nullptr || f->hs == nullptr || f->ys == nullptr)
      return DSCA_ERR_BAD_ARG;
    if (f->shared_n1p <= 0 || f->shared_n1p % 256 != 0 ||
        f->shared_ip != (glu ? f->shared_n1p / 2 : f->shared_n1p))
      return DSCA_ERR_BAD_ARG;
  }
  int num_sms = 0, major = 0;
  int rc = device_info(&num_sms, &major);
  if (rc) return rc;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (f->dtype == DSCA_BF16) {
    if (major != 10) return DSCA_ERR_UNSUPPORTED;
    if (f->d < 64) return DSCA_ERR_BAD_ARG;  // one 64-wide K box at least
    const void* ptrs[] = {f->a, f->w1, f->w2, f->h, f->y};
    for (const void* p : ptrs)
      if (!aligned16(p)) return DSCA_ERR_BAD_ARG;
    return dsca::launch_grouped_ffn_bf16(f, num_sms, st);
  }
  if (f->dtype == DSCA_F8E4M3) {
    if (major != 10) return DSCA_ERR_UNSUPPORTED;
    if (f->ep_ctx != nullptr) return DSCA_ERR_UNSUPPORTED;  // fused return epilogue: bf16 path only
    if (f->d < 64 || f->w1_scale == nullptr || f->w2_scale == nullptr) return DSCA_ERR_BAD_ARG;
    if (f->shared_rows > 0 && (f->ws1_scale == nullptr || f->ws2_scale == nullptr)) return DSCA_ERR_BAD_ARG;
    const void* ptrs[] = {f->a, f->w1, f->w2, f->h, f->y};
    for (const void* p : ptrs)
      if (!aligned16(p)) return DSCA_ERR_BAD_ARG;
    if (f->f8_split) {
      // e4m3 weights as they are, tokens as two e4m3 terms (CTA-pair kind::f8f6f4 tiles)
      if (f->a_scale == nullptr || f->hq == nullptr || f->h_scale == nullptr || !aligned16(f->hq))
        return DSCA_ERR_BAD_ARG;
      if (f->shared_rows > 0 && (f->xs_scale == nullptr || f->hsq == nullptr || f->hs_scale == nullptr ||
                                 !aligned16(f->xs) || !aligned16(f->hsq) || !aligned16(f->hs)))
        return DSCA_ERR_BAD_ARG;
      return dsca::launch_grouped_ffn_f8_split(f, num_sms, st);
    }
    // tile_rows 256: weights converted into tensor memory (swap-AB); otherwise through shared memory
    if (f->tile_rows == 256) return dsca::launch_grouped_ffn_fp8_tmem(f, num_sms, st);
    return dsca::launch_grouped_ffn_fp8(f, num_sms, st);
  }
  if (f->dtype == DSCA_F32) {
    if (f->ep_ctx != nullptr) return DSCA_ERR_UNSUPPORTED;  // the fused return path is bf16 only
    return dsca::launch_grouped_ffn_f32(f, num_sms, st);
  }
  return DSCA_ERR_BAD_ARG;
}

int dsca_combine(const dsca_combine_args* a, dsca_stream_t stream) {
  if (a == nullptr || a->y == nullptr || a->token_row == nullptr || a->topk_w == nullptr ||
      a->out == nullptr || a->T < 0 || a->d <= 0 || a->top_k <= 0 || a->top_k > DSCA_MAX_TOPK)
    return DSCA_ERR_BAD_ARG;
  if (a->dtype != DSCA_BF16 && a->dtype != DSCA_F32) return DSCA_ERR_BAD_ARG;
  if (a->d % 8 != 0 || !aligned16(a->y) || !aligned16(a->out) || (a->ys && !aligned16(a->ys)))
    return DSCA_ERR_BAD_ARG;
  if ((a->ys == nullptr) != (a->shared_gate == nullptr)) return DSCA_ERR_BAD_ARG;
  return dsca::launch_combine(a, reinterpret_cast<cudaStream_t>(stream));
}

int dsca_qos_priority(const dsca_qos_args* a, dsca_stream_t stream) {
  if (a == nullptr || a->x == nullptr || a->logits == nullptr || a->topk_ids == nullptr ||
      a->token_score == nullptr || a->expert_priority == nullptr || a->T < 0 || a->d <= 0 || a->E <= 0 ||
      a->top_k <= 0 || a->top_k > DSCA_MAX_TOPK || a->top_k > a->E)
    return DSCA_ERR_BAD_ARG;
  if (a->dtype != DSCA_BF16 && a->dtype != DSCA_F32) return DSCA_ERR_BAD_ARG;
  if (a->attention_mode != 0 && a->attention_mode != 1) return DSCA_ERR_BAD_ARG;
  if (a->E > 4 * DSCA_MAX_EXPERTS) return DSCA_ERR_CAPACITY;
  if ((a->partial == nullptr) != (a->done_counter == nullptr)) return DSCA_ERR_BAD_ARG;
  if (a->top_k > DSCA_MAX_TOPK) return DSCA_ERR_BAD_ARG;
  return dsca::launch_qos(a, reinterpret_cast<cudaStream_t>(stream));
}

int dsca_check_error(int32_t* err_dev, dsca_stream_t stream) {
  if (err_dev == nullptr) return DSCA_ERR_BAD_ARG;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  int32_t h = 0;
  if (cudaMemcpyAsync(&h, err_dev, sizeof(int32_t), cudaMemcpyDeviceToHost, st) != cudaSuccess)
    return DSCA_ERR_CUDA;
  if (cudaStreamSynchronize(st) != cudaSuccess) return DSCA_ERR_CUDA;
  if (h != 0) {
    if (cudaMemsetAsync(err_dev, 0, sizeof(int32_t), st) != cudaSuccess) return DSCA_ERR_CUDA;
    if (cudaStreamSynchronize(st) != cudaSuccess) return DSCA_ERR_CUDA;
  }
  switch (h) {
    case dsca::kErrNone: return DSCA_OK;
    case dsca::kErrWaitTimeout: return DSCA_ERR_WAIT_TIMEOUT;
    case dsca::kErrIndex: return DSCA_ERR_DEVICE_INDEX;
    case dsca::kErrCapacity: return DSCA_ERR_CAPACITY;
    default: return DSCA_ERR_DEVICE_INDEX;
  }
}

int dsca_exp_neg_eval(const float* x, float* y, int n, dsca_stream_t stream) {
  if ((x == nullptr || y == nullptr) && n > 0) return DSCA_ERR_BAD_ARG;
  return dsca::launch_exp_eval(x, y, n, reinterpret_cast<cudaStream_t>(stream));
}

}  // extern "C"
