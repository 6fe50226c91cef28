// K3 dispatch scan + permute, and K6 combine.
//
// Scan: counts, expert-major offsets and per-block base ranks from the router's per-block
// histograms (replaces bincount / sort / nonzero at src/qosmoe/moe_layer.py:206-215,300-304
// and qwen_ep_adapter/qwen_ep.py:62,69,80).
// Permute: stable expert-major (or plan-ordered send-buffer) row copy, one warp per routed
// (token, slot), 16-byte vector loads / stores (replaces the gathers of
// src/qosmoe/moe_layer.py:214-215 and Scheduler.distribute_tokens,
// src/harmonymoe/scheduler.py:101-124).
// Combine: deterministic gather-reduce (replaces router_probs * h at moe_layer.py:255-258 and
// index_add_ + shared add at qwen_ep.py:92-94).
#include "common.cuh"
#include "fp8_split.cuh"

namespace dsca {

// ------------------------------------------------------------------ scan
// One CTA of 1024 threads: thread (e, c) with c in [0, 16) sums a contiguous run of blocks of
// expert e, the 16 partials are scanned in shared memory, then each thread writes the base
// ranks of its run.
constexpr int kScanChunks = 16;

__global__ void __launch_bounds__(1024) scan_kernel(const int32_t* __restrict__ hist, int nb, int E,
                                                    int32_t* counts, int32_t* offsets,
                                                    int32_t* block_base) {
  __shared__ int part[DSCA_MAX_EXPERTS * 4][kScanChunks + 1];
  __shared__ int cnt_s[DSCA_MAX_EXPERTS * 4];
  const int per = (nb + kScanChunks - 1) / kScanChunks;
  for (int base_e = 0; base_e < E; base_e += 1024 / kScanChunks) {
    int e = base_e + threadIdx.x / kScanChunks;
    int c = threadIdx.x % kScanChunks;
    int b0 = c * per, b1 = min(nb, b0 + per);
    int s = 0;
    if (e < E)
      for (int b = b0; b < b1; ++b) s += hist[(size_t)b * E + e];
    if (e < E) part[e][c] = s;
    __syncthreads();
    if (e < E && c == 0) {
      int run = 0;
      for (int i = 0; i < kScanChunks; ++i) {
        int v = part[e][i];
        part[e][i] = run;
        run += v;
      }
      cnt_s[e] = run;
      counts[e] = run;
    }
    __syncthreads();
    if (e < E) {
      int run = part[e][c];
      for (int b = b0; b < b1; ++b) {
        int v = hist[(size_t)b * E + e];
        block_base[(size_t)b * E + e] = run;
        run += v;
      }
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    int run = 0;
    for (int e = 0; e < E; ++e) {
      offsets[e] = run;
      run += cnt_s[e];
    }
    offsets[E] = run;
  }
}

int launch_scan(const dsca_scan_args* a, cudaStream_t stream) {
  scan_kernel<<<1, 1024, 0, stream>>>(a->block_hist, a->nblocks, a->E, a->counts, a->offsets,
                                      a->block_base);
  return cudaGetLastError() == cudaSuccess ? DSCA_OK : DSCA_ERR_CUDA;
}

// ------------------------------------------------------------------ permute
// One warp per (token, slot) assignment, grid-stride over the assignments with a grid that is
// resident at once (two CTAs per SM): every CTA starts immediately, so the programmatic
// dependent launch below fires at the start and leaves room on each SM for the dependent GEMM.
template <int ESZ>
__device__ __forceinline__ void permute_one(const dsca_permute_args& a, int w, int lane) {
  const int t = w / a.top_k;
  const int e = a.topk_ids[w];
  if (e < 0 || e >= a.E) {
    if (lane == 0) record_error(a.err, kErrIndex);
    return;
  }
  const int b = t / DSCA_ROUTER_TOKENS;
  const int q = a.block_base[(size_t)b * a.E + e] + a.local_rank[w];
  int row;
  if (a.cum_split == nullptr) {
    row = a.offsets[e] + q;
  } else {
    int dst = 0;
    int before = 0;
    const int32_t* cs = a.cum_split + (size_t)e * a.G;
    while (dst < a.G && q >= cs[dst]) ++dst;
    if (dst >= a.G) {
      if (lane == 0) record_error(a.err, kErrIndex);
      return;
    }
    before = dst > 0 ? cs[dst - 1] : 0;
    row = a.dest_base[(size_t)e * a.G + dst] + (q - before);
  }
  if (row < 0 || row >= a.capacity) {
    if (lane == 0) record_error(a.err, kErrCapacity);
    return;
  }
  if (lane == 0) a.token_row[w] = row;
  if (ESZ == 2 && a.out_e4m3) {
    // two e4m3 terms per value (fp8_split.cuh); the copy of x for the shared expert is written
    // once per token, by its slot-0 warp
    const int Kp = (a.d + 127) & ~127;
    const uint16_t* xr = reinterpret_cast<const uint16_t*>(a.x) + (size_t)t * a.d;
    uint8_t* dst = reinterpret_cast<uint8_t*>(a.out) + (size_t)row * 2 * Kp;
    uint8_t* dq = (a.x_q != nullptr && (w % a.top_k) == 0)
                      ? reinterpret_cast<uint8_t*>(a.x_q) + (size_t)t * 2 * Kp
                      : nullptr;
    const float inv = f8s::split_row(xr, a.d, Kp, dst, dq, lane);
    if (lane == 0) {
      a.out_scale[row] = inv;
      if (dq != nullptr) a.x_scale[t] = inv;
    }
    return;
  }
  const size_t row_bytes = (size_t)a.d * ESZ;
  const uint4* src = reinterpret_cast<const uint4*>(reinterpret_cast<const char*>(a.x) + (size_t)t * row_bytes);
  uint4* dstp = reinterpret_cast<uint4*>(reinterpret_cast<char*>(a.out) + (size_t)row * row_bytes);
  const int nvec = (int)(row_bytes / 16);
  if (ESZ == 2 && a.out_f16) {
    // bf16 -> f16 on the way (operand of the fp8-weight FFN); the f16 copy of x for the shared
    // expert is written once per token, by its slot-0 warp
    uint4* xh = (a.x_f16 != nullptr && (w % a.top_k) == 0)
                    ? reinterpret_cast<uint4*>(reinterpret_cast<char*>(a.x_f16) + (size_t)t * row_bytes)
                    : nullptr;
    for (int v = lane; v < nvec; v += 32) {
      const uint4 u = src[v];
      const __nv_bfloat162* bb = reinterpret_cast<const __nv_bfloat162*>(&u);
      uint4 o;
      uint32_t* op = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = __bfloat1622float2(bb[i]);
        __half2 h = __floats2half2_rn(f.x, f.y);
        op[i] = *reinterpret_cast<uint32_t*>(&h);
      }
      dstp[v] = o;
      if (xh != nullptr) xh[v] = o;
    }
  } else {
    // eight 16-byte loads in flight per lane before the stores (one memory latency per row)
    int v = lane;
    for (; v + 7 * 32 < nvec; v += 8 * 32) {
      uint4 r[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) r[i] = src[v + 32 * i];
#pragma unroll
      for (int i = 0; i < 8; ++i) dstp[v + 32 * i] = r[i];
    }
    for (; v < nvec; v += 32) dstp[v] = src[v];
  }
}

template <int ESZ>
__global__ void __launch_bounds__(256) permute_kernel(dsca_permute_args a) {
  // a GEMM1 launched as a programmatic dependent may start its shared-expert tiles now; it
  // waits for this grid before reading the permuted rows
  pdl_launch_dependents();
  const int lane = lane_id();
  const int total = a.T * a.top_k;
  const int nwarps = (int)(gridDim.x * (blockDim.x >> 5));
  for (int w = (int)((blockIdx.x * blockDim.x + threadIdx.x) >> 5); w < total; w += nwarps)
    permute_one<ESZ>(a, w, lane);
}

// dsca_split_rows: one warp per row, grid-stride over the rows.
__global__ void __launch_bounds__(256) split_rows_kernel(dsca_split_args a) {
  const int lane = lane_id();
  int rows = a.rows;
  if (a.rows_dev != nullptr) rows = min(rows, max(0, *a.rows_dev));
  const int Kp = (a.K + 127) & ~127;
  const int nwarps = (int)(gridDim.x * (blockDim.x >> 5));
  for (int r = (int)((blockIdx.x * blockDim.x + threadIdx.x) >> 5); r < rows; r += nwarps) {
    const uint16_t* src = reinterpret_cast<const uint16_t*>(a.src) + (size_t)r * a.ld;
    uint8_t* dst = reinterpret_cast<uint8_t*>(a.dst) + (size_t)r * 2 * Kp;
    const float inv = f8s::split_row(src, a.K, Kp, dst, nullptr, lane);
    if (lane == 0) a.inv_scale[r] = inv;
  }
}

int launch_split_rows(const void* src, int ld, int rows, const int32_t* rows_dev, int K, void* dst, float* inv_scale,
                      cudaStream_t stream) {
  if (rows <= 0) return DSCA_OK;
  const int num_sms = current_device_sms();
  if (num_sms == 0) return DSCA_ERR_CUDA;
  dsca_split_args a;
  a.src = src;
  a.ld = ld;
  a.rows = rows;
  a.K = K;
  a.rows_dev = rows_dev;
  a.dst = dst;
  a.inv_scale = inv_scale;
  const long long need = ((long long)rows * 32 + 255) / 256;
  const int blocks = (int)(need < 4LL * num_sms ? need : 4LL * num_sms);
  split_rows_kernel<<<blocks, 256, 0, stream>>>(a);
  return cudaGetLastError() == cudaSuccess ? DSCA_OK : DSCA_ERR_CUDA;
}

int launch_permute(const dsca_permute_args* a, cudaStream_t stream) {
  const long long warps = (long long)a->T * a->top_k;
  if (warps == 0) return DSCA_OK;
  const int num_sms = current_device_sms();
  if (num_sms == 0) return DSCA_ERR_CUDA;
  // the SMs keep their full shared-memory carveout while the permute runs, so that the
  // dependent GEMM's CTAs can be placed next to it
  static PerDeviceOnce carveout_once;
  carveout_once.run([] {
    cudaFuncSetAttribute(permute_kernel<2>, cudaFuncAttributePreferredSharedMemoryCarveout,
                         (int)cudaSharedmemCarveoutMaxShared);
    cudaFuncSetAttribute(permute_kernel<4>, cudaFuncAttributePreferredSharedMemoryCarveout,
                         (int)cudaSharedmemCarveoutMaxShared);
    cudaGetLastError();
    return cudaSuccess;
  });
  // two 256-thread CTAs per SM (46 registers a thread): resident together, with room left on every
  // SM for one CTA of the dependent GEMM (192 threads, 123 registers, 197 KB shared memory)
  const long long need = (warps * 32 + 255) / 256;
  const int blocks = (int)(need < 2LL * num_sms ? need : 2LL * num_sms);
  if (a->dtype == DSCA_BF16)
    permute_kernel<2><<<blocks, 256, 0, stream>>>(*a);
  else
    permute_kernel<4><<<blocks, 256, 0, stream>>>(*a);
  return cudaGetLastError() == cudaSuccess ? DSCA_OK : DSCA_ERR_CUDA;
}

// ------------------------------------------------------------------ combine
// One warp per token; lane owns 8 consecutive columns per step (one 16-byte bf16 vector or
// two 16-byte f32 vectors).  Sum order: slot 0..k-1, then the shared expert.
template <typename T>
struct Vec8;
template <>
struct Vec8<__nv_bfloat16> {
  struct Raw {
    uint4 u;
  };
  static __device__ Raw load_raw(const void* p) { return Raw{*reinterpret_cast<const uint4*>(p)}; }
  static __device__ void convert(const Raw& r, float (&v)[8]) {
    const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(&r.u);
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = __bfloat162float(h[i]);
  }
  static __device__ void load(const void* p, float (&v)[8]) {
    uint4 u = *reinterpret_cast<const uint4*>(p);
    const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(&u);
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = __bfloat162float(h[i]);
  }
  static __device__ void store(void* p, const float (&v)[8]) {
    uint4 u;
    u.x = pack_bf16x2(v[0], v[1]);
    u.y = pack_bf16x2(v[2], v[3]);
    u.z = pack_bf16x2(v[4], v[5]);
    u.w = pack_bf16x2(v[6], v[7]);
    *reinterpret_cast<uint4*>(p) = u;
  }
};
template <>
struct Vec8<float> {
  struct Raw {
    float4 a, b;
  };
  static __device__ Raw load_raw(const void* p) {
    return Raw{reinterpret_cast<const float4*>(p)[0], reinterpret_cast<const float4*>(p)[1]};
  }
  static __device__ void convert(const Raw& r, float (&v)[8]) {
    v[0] = r.a.x; v[1] = r.a.y; v[2] = r.a.z; v[3] = r.a.w;
    v[4] = r.b.x; v[5] = r.b.y; v[6] = r.b.z; v[7] = r.b.w;
  }
  static __device__ void load(const void* p, float (&v)[8]) {
    float4 a = reinterpret_cast<const float4*>(p)[0];
    float4 b = reinterpret_cast<const float4*>(p)[1];
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  }
  static __device__ void store(void* p, const float (&v)[8]) {
    reinterpret_cast<float4*>(p)[0] = make_float4(v[0], v[1], v[2], v[3]);
    reinterpret_cast<float4*>(p)[1] = make_float4(v[4], v[5], v[6], v[7]);
  }
};

// KC: the slot count as a compile-time constant (1, 2, 4, 8), or 0 for any count up to
// DSCA_MAX_TOPK (registers sized for the maximum).
template <typename T, int KC>
__global__ void __launch_bounds__(256) combine_kernel(dsca_combine_args a) {
  constexpr int KMAX = KC > 0 ? KC : DSCA_MAX_TOPK;
  pdl_wait();  // launched as a programmatic dependent of GEMM2: its outputs are complete past here
  const int t = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = lane_id();
  if (t >= a.T) return;
  int rows[KMAX];
  float w[KMAX];
  bool bad = false;
#pragma unroll
  for (int j = 0; j < KMAX; ++j) {
    if (KC > 0 || j < a.top_k) {
      rows[j] = a.token_row[(size_t)t * a.top_k + j];
      w[j] = a.topk_w[(size_t)t * a.top_k + j];
      bad |= rows[j] < 0 || rows[j] >= a.rows;
    }
  }
  if (bad) {
    if (lane == 0) record_error(a.err, kErrIndex);
    return;
  }
  const float sg = (a.ys != nullptr && a.shared_gate != nullptr) ? a.shared_gate[t] : 0.0f;
  const T* Y = reinterpret_cast<const T*>(a.y);
  const T* YS = reinterpret_cast<const T*>(a.ys);
  T* O = reinterpret_cast<T*>(a.out);
  // every slot's 16-byte piece (and the shared expert's) of two chunks is loaded before the first
  // FMA, so two chunks cost one memory latency; the sums still run in slot order, then the
  // shared term
  using R = typename Vec8<T>::Raw;
  constexpr int U = 2;  // chunks in flight per lane
  for (int c0 = lane * 8; c0 < a.d; c0 += 256 * U) {
    R raw[U][KMAX + 1];
#pragma unroll
    for (int h = 0; h < U; ++h) {
      const int c = c0 + 256 * h;
      if (c < a.d) {
#pragma unroll
        for (int j = 0; j < KMAX; ++j)
          if (KC > 0 || j < a.top_k) raw[h][j] = Vec8<T>::load_raw(Y + (size_t)rows[j] * a.d + c);
        if (YS != nullptr) raw[h][KMAX] = Vec8<T>::load_raw(YS + (size_t)t * a.d + c);
      }
    }
#pragma unroll
    for (int h = 0; h < U; ++h) {
      const int c = c0 + 256 * h;
      if (c >= a.d) break;
      float acc[8], v[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] = 0.0f;
#pragma unroll
      for (int j = 0; j < KMAX; ++j) {
        if (KC > 0 || j < a.top_k) {
          Vec8<T>::convert(raw[h][j], v);
#pragma unroll
          for (int i = 0; i < 8; ++i) acc[i] = __fmaf_rn(w[j], v[i], acc[i]);
        }
      }
      if (YS != nullptr) {
        Vec8<T>::convert(raw[h][KMAX], v);
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[i] = __fmaf_rn(sg, v[i], acc[i]);
      }
      Vec8<T>::store(O + (size_t)t * a.d + c, acc);
    }
  }
}


template <typename T, int KC>
static void launch_combine_k(const dsca_combine_args& a, int blocks, cudaStream_t stream) {
  if (!a.pdl) {
    combine_kernel<T, KC><<<blocks, 256, 0, stream>>>(a);
    return;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)blocks);
  cfg.blockDim = dim3(256);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaLaunchKernelEx(&cfg, combine_kernel<T, KC>, a);
}

template <typename T>
static void launch_combine(const dsca_combine_args& a, int blocks, cudaStream_t stream) {
  switch (a.top_k) {
    case 1: launch_combine_k<T, 1>(a, blocks, stream); break;
    case 2: launch_combine_k<T, 2>(a, blocks, stream); break;
    case 4: launch_combine_k<T, 4>(a, blocks, stream); break;
    case 8: launch_combine_k<T, 8>(a, blocks, stream); break;
    default: launch_combine_k<T, 0>(a, blocks, stream); break;
  }
}

int launch_combine(const dsca_combine_args* a, cudaStream_t stream) {
  if (a->T == 0) return DSCA_OK;
  const int blocks = (int)(((long long)a->T * 32 + 255) / 256);
  if (a->dtype == DSCA_BF16)
    launch_combine<__nv_bfloat16>(*a, blocks, stream);
  else
    launch_combine<float>(*a, blocks, stream);
  return cudaGetLastError() == cudaSuccess ? DSCA_OK : DSCA_ERR_CUDA;
}

}  // namespace dsca
