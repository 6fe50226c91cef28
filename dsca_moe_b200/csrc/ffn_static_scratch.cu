// Grouped expert FFN for callers that cannot allocate device memory.
//
// dsca_grouped_ffn needs an intermediate buffer (the activated GEMM1 output, `h` / `hs`) that
// the caller allocates.  Some callers cannot do that: code running inside a CUDA-graph replay
// or a driver/runtime callback, an embedding host whose memory is owned by a foreign allocator
// with no free capacity, or a process whose allocator is frozen after start-up.  For them,
// dsca_grouped_ffn_static_scratch keeps the intermediate in a fixed array compiled into this
// library instead.  The caller still passes the inputs and the outputs.
//
// Costs and rules:
//   * every GPU that loads this library holds DSCA_STATIC_SCRATCH_BYTES (16 MiB) of device
//     memory for the array until the process exits;
//   * the first call on a device looks up the array's device address (cudaGetSymbolAddress)
//     with that device current; make that first call before any stream capture.  The address
//     is cached per device and per CUDA context (its unique id), so after a cudaDeviceReset the
//     next call looks it up again in the new context;
//   * bf16 (tcgen05) and f32 (CUDA cores) only: fp8-e4m3 weights and, for f32, the fused
//     expert-parallel return (ep_ctx) are refused with DSCA_ERR_UNSUPPORTED, as
//     dsca_grouped_ffn does for f32;
//   * all calls share the one array: two calls whose work overlaps on the GPU (different
//     streams, or different host threads on the same device) race on it and produce garbage;
//     calls that are ordered on one stream are safe.  The array keeps the previous call's
//     contents; nothing in it has to start at zero, because GEMM1 writes every element that
//     GEMM2 reads back for a valid output row.
#include <mutex>

#include "common.cuh"

namespace dsca {
int launch_grouped_ffn_bf16(const dsca_ffn_args* f, int num_sms, cudaStream_t stream);
int launch_grouped_ffn_f32(const dsca_ffn_args* f, int num_sms, cudaStream_t stream);
}  // namespace dsca

namespace {

static __device__ __align__(256) unsigned char g_ffn_scratch[DSCA_STATIC_SCRATCH_BYTES];

void* g_scratch_addr[dsca::kMaxDevices] = {};
unsigned long long g_ctx_id[dsca::kMaxDevices] = {};
int g_num_sms[dsca::kMaxDevices] = {};
int g_major[dsca::kMaxDevices] = {};
std::mutex g_setup_mutex;

// Unique id of the current CUDA context (0 when it cannot be read): a context created after a
// device reset gets a new id even if its handle value is reused.
unsigned long long current_context_id() {
  typedef CUresult (*GetCurrent)(CUcontext*);
  typedef CUresult (*GetId)(CUcontext, unsigned long long*);
  static GetCurrent get_current = nullptr;
  static GetId get_id = nullptr;
  if (get_current == nullptr || get_id == nullptr) {
    void* p = nullptr;
    void* q = nullptr;
    cudaDriverEntryPointQueryResult r1, r2;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &r1) != cudaSuccess ||
        r1 != cudaDriverEntryPointSuccess ||
        cudaGetDriverEntryPoint("cuCtxGetId", &q, cudaEnableDefault, &r2) != cudaSuccess ||
        r2 != cudaDriverEntryPointSuccess)
      return 0;
    get_current = reinterpret_cast<GetCurrent>(p);
    get_id = reinterpret_cast<GetId>(q);
  }
  CUcontext ctx = nullptr;
  unsigned long long id = 0;
  if (get_current(&ctx) != CUDA_SUCCESS || ctx == nullptr || get_id(ctx, &id) != CUDA_SUCCESS) return 0;
  return id;
}

// Once per device and context, with that device current: the array's device address and the
// SM count.
int scratch_setup(int dev, void** addr, int* num_sms, int* major) {
  if (dev < 0 || dev >= dsca::kMaxDevices) return DSCA_ERR_CUDA;
  std::lock_guard<std::mutex> lock(g_setup_mutex);
  const unsigned long long ctx_id = current_context_id();
  if (g_scratch_addr[dev] == nullptr || ctx_id != g_ctx_id[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_ffn_scratch) != cudaSuccess || p == nullptr) return DSCA_ERR_CUDA;
    cudaDeviceProp prop;
    if (cudaGetDeviceProperties(&prop, dev) != cudaSuccess) return DSCA_ERR_CUDA;
    g_num_sms[dev] = prop.multiProcessorCount;
    g_major[dev] = prop.major;
    g_scratch_addr[dev] = p;
    g_ctx_id[dev] = current_context_id();  // read again: the lookup may have created the context
  }
  *addr = g_scratch_addr[dev];
  *num_sms = g_num_sms[dev];
  *major = g_major[dev];
  return DSCA_OK;
}

size_t align256(size_t n) { return (n + 255) & ~size_t(255); }

}  // namespace

extern "C" int dsca_grouped_ffn_static_scratch(const dsca_ffn_args* a, dsca_stream_t stream) {
  if (a == nullptr || a->a == nullptr || a->w1 == nullptr || a->w2 == nullptr || a->y == nullptr ||
      a->group_offsets == nullptr)
    return DSCA_ERR_BAD_ARG;
  if (a->h != nullptr || a->hs != nullptr) return DSCA_ERR_BAD_ARG;  // the scratch is internal
  if (a->shared_handoff != 0 && a->shared_handoff != 1) return DSCA_ERR_BAD_ARG;
  if (a->num_groups <= 0 || a->num_groups > 256 || a->capacity < 0 || a->d <= 0 || a->num_experts_w <= 0)
    return a->num_groups > 256 ? DSCA_ERR_CAPACITY : DSCA_ERR_BAD_ARG;
  if (a->act != DSCA_ACT_RELU && a->act != DSCA_ACT_SWIGLU) return DSCA_ERR_BAD_ARG;
  const bool glu = a->act == DSCA_ACT_SWIGLU;
  if (a->n1p <= 0 || a->n1p % 256 != 0 || a->dp < a->d || a->dp % 256 != 0 || a->d % 8 != 0 ||
      a->ip != (glu ? a->n1p / 2 : a->n1p))
    return DSCA_ERR_BAD_ARG;
  if (a->shared_rows > 0 &&
      (a->xs == nullptr || a->ws1 == nullptr || a->ws2 == nullptr || a->ys == nullptr || a->shared_n1p <= 0 ||
       a->shared_n1p % 256 != 0 || a->shared_ip != (glu ? a->shared_n1p / 2 : a->shared_n1p)))
    return DSCA_ERR_BAD_ARG;
  if (a->dtype == DSCA_F8E4M3) return DSCA_ERR_UNSUPPORTED;  // fp8 weights: dsca_grouped_ffn only
  if (a->dtype != DSCA_BF16 && a->dtype != DSCA_F32) return DSCA_ERR_BAD_ARG;
  if (a->dtype == DSCA_F32 && a->ep_ctx != nullptr) return DSCA_ERR_UNSUPPORTED;  // as dsca_grouped_ffn
  if (a->phases != 0 && a->phases != 3) return DSCA_ERR_BAD_ARG;  // GEMM2 needs this call's GEMM1
  const void* vec_ptrs[] = {a->a, a->w1, a->w2, a->y, a->xs, a->ws1, a->ws2, a->ys};
  for (const void* p : vec_ptrs)
    if ((reinterpret_cast<uintptr_t>(p) & 15u) != 0) return DSCA_ERR_BAD_ARG;

  // size check before touching the device
  const size_t esz = a->dtype == DSCA_BF16 ? 2 : 4;
  const size_t h_bytes = align256((size_t)a->capacity * (size_t)a->ip * esz);
  const size_t hs_bytes = a->shared_rows > 0 ? (size_t)a->shared_rows * (size_t)a->shared_ip * esz : 0;
  if (h_bytes + hs_bytes > (size_t)DSCA_STATIC_SCRATCH_BYTES) return DSCA_ERR_CAPACITY;

  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return DSCA_ERR_CUDA;
  void* base = nullptr;
  int num_sms = 0, major = 0;
  int rc = scratch_setup(dev, &base, &num_sms, &major);
  if (rc) return rc;

  dsca_ffn_args f = *a;
  f.h = base;
  f.hs = a->shared_rows > 0 ? static_cast<void*>(static_cast<unsigned char*>(base) + h_bytes) : nullptr;
  f.phases = 3;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (f.dtype == DSCA_BF16) {
    if (major != 10) return DSCA_ERR_UNSUPPORTED;
    if (f.d < 64) return DSCA_ERR_BAD_ARG;
    return dsca::launch_grouped_ffn_bf16(&f, num_sms, st);
  }
  return dsca::launch_grouped_ffn_f32(&f, num_sms, st);
}
