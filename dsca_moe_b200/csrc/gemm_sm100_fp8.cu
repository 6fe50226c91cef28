// K5 (fp8-e4m3 expert weights) — grouped GEMM with e4m3 weights and per-output-channel fp32
// scales on the 5th-generation tensor cores (sm_100a).
//
// Activations (the permuted rows, the shared-expert input and the GEMM1 intermediate) are f16
// here: every e4m3 value is exactly an f16, so one `cvt.rn.f16x2.e4m3x2` turns two weights into
// MMA operands, and the MMA is tcgen05 kind::f16 (f16 x f16, fp32 accumulate).  The per-channel
// scale multiplies the fp32 accumulator in the epilogue: y_c = s_c * sum_k a_k q_ck.
// Weight bytes read from HBM halve against bf16.
//
// Pipeline per 128 x 256 x 64 step (3 stages of 64 KB):
//   warp 0      TMA: A tile (f16, 128-byte swizzle) + the e4m3 weight tile (row-major staging)
//   warps 6-9   convert the staged e4m3 tile to f16 in the 128-byte-swizzled K-major layout the
//               MMA reads, fence the generic-proxy stores for the async proxy, arrive
//   warp 1      TMEM allocation; one thread issues 4 x tcgen05.mma (M128 N256 K16) per stage
//   warps 2-5   epilogue: TMEM -> registers, x scale, SiLU(g)*u (GEMM1, f16 out) or store
//               (GEMM2, bf16 out)
// Same tile enumeration, bounded waits and abort path as the bf16 kernel.  No TMA multicast.
#include "common.cuh"

namespace dsca {
namespace gemm8 {

constexpr int BM = 128, BN = 256, BK = 64;
constexpr int kStages = 3;
constexpr int kABytes = BM * BK * 2;   // f16 A tile
constexpr int kBBytes = BN * BK * 2;   // f16 B tile (converted)
constexpr int kB8Bytes = BN * BK;      // e4m3 B tile (staging)
constexpr int kThreads = 320;
constexpr int kTmemCols = 512;
constexpr int kMaxGroups = 256;
constexpr int kSmemBytes = kStages * (kABytes + kBBytes + kB8Bytes) + 1024;

enum Epi { kEpiSwiGLU = 0, kEpiReLU = 1, kEpiStore = 2 };

struct Segment {
  const int32_t* group_offsets;
  const int32_t* group_weight;
  int ngroups, rows, n_tiles, b_rows_per_group, k_blocks;
  void* c;              // f16 (GEMM1) or bf16 (GEMM2)
  int ldc, n_store, capacity;
  const float* scale;   // per B row (output channel)
};

struct Params {
  Segment seg[2];
  int nseg, epi;
  int32_t* err;
};

struct TileInfo {
  int seg, row0, rows_valid, b_row0, n_blk;
};

struct SmemCtl {
  uint64_t full[kStages];
  uint64_t bready[kStages];
  uint64_t empty[kStages];
  uint64_t tmem_full[2];
  uint64_t tmem_empty[2];
  uint64_t mma_done;
  uint32_t tmem_base;
  int abort_flag;
  int total_tiles, seg0_tiles;
  int tile_start[kMaxGroups + 1];
  int goff[kMaxGroups + 1];
  int gw[kMaxGroups];
};

__device__ __forceinline__ TileInfo decode(const Params& p, const SmemCtl& s, int tile) {
  TileInfo ti;
  if (tile < s.seg0_tiles) {
    const Segment& sg = p.seg[0];
    int lo = 0, hi = sg.ngroups;
    while (hi - lo > 1) {
      int mid = (lo + hi) >> 1;
      if (s.tile_start[mid] <= tile) lo = mid; else hi = mid;
    }
    int local = tile - s.tile_start[lo];
    int m_blk = local / sg.n_tiles;
    ti.n_blk = local - m_blk * sg.n_tiles;
    ti.seg = 0;
    ti.row0 = s.goff[lo] + m_blk * BM;
    ti.rows_valid = min(BM, s.goff[lo + 1] - s.goff[lo] - m_blk * BM);
    ti.b_row0 = s.gw[lo] * sg.b_rows_per_group + ti.n_blk * BN;
  } else {
    const Segment& sg = p.seg[1];
    int local = tile - s.seg0_tiles;
    int m_blk = local / sg.n_tiles;
    ti.n_blk = local - m_blk * sg.n_tiles;
    ti.seg = 1;
    ti.row0 = m_blk * BM;
    ti.rows_valid = min(BM, sg.rows - ti.row0);
    ti.b_row0 = ti.n_blk * BN;
  }
  return ti;
}

__device__ __forceinline__ void mbar_drain(uint32_t bar, uint32_t parity) {
  const uint64_t t0 = globaltimer_ns();
  while (!mbar_try_wait(bar, parity))
    if (globaltimer_ns() - t0 > kWaitLimitNs) return;
}

__device__ __forceinline__ float silu(float g) { return g / (1.0f + __expf(-g)); }

__device__ __forceinline__ uint32_t e4m3x2_to_f16x2(uint16_t v) {
  uint32_t r;
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(r) : "h"(v));
  return r;
}

__device__ __forceinline__ uint32_t pack_f16x2(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

// Instruction descriptor, kind::f16: A = B = f16, D = f32, both K-major.
__host__ __device__ constexpr uint32_t idesc_f16_f32(int M, int N) {
  return (1u << 4) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

template <int EPI>
__global__ void __launch_bounds__(kThreads, 1)
    grouped_gemm_fp8_kernel(const __grid_constant__ CUtensorMap tmA0, const __grid_constant__ CUtensorMap tmB0,
                            const __grid_constant__ CUtensorMap tmA1, const __grid_constant__ CUtensorMap tmB1,
                            const Params p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  __shared__ SmemCtl ctl;
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t smem_a = smem_u32(smem);
  const uint32_t smem_b = smem_a + kStages * kABytes;
  const uint32_t smem_b8 = smem_b + kStages * kBBytes;
  uint8_t* b8_ptr = smem + kStages * (kABytes + kBBytes);
  uint8_t* b16_ptr = smem + kStages * kABytes;

  const int warp = warp_id(), lane = lane_id();
  volatile int* abort_flag = &ctl.abort_flag;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(smem_u32(&ctl.full[s]), 1);
      mbar_init(smem_u32(&ctl.bready[s]), 128);
      mbar_init(smem_u32(&ctl.empty[s]), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(smem_u32(&ctl.tmem_full[a]), 1);
      mbar_init(smem_u32(&ctl.tmem_empty[a]), 128);
    }
    mbar_init(smem_u32(&ctl.mma_done), 1);
    ctl.abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmA0);
    prefetch_tmap(&tmB0);
    if (p.nseg > 1) {
      prefetch_tmap(&tmA1);
      prefetch_tmap(&tmB1);
    }
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(&ctl.tmem_base), kTmemCols);
    tmem_relinquish();
  }
  if (warp == 2) {
    const Segment& sg = p.seg[0];
    const int ng = sg.ngroups;
    for (int g = lane; g <= ng; g += 32)
      ctl.goff[g] = sg.group_offsets ? sg.group_offsets[g] : (g == 0 ? 0 : sg.rows);
    for (int g = lane; g < ng; g += 32) ctl.gw[g] = sg.group_weight ? sg.group_weight[g] : g;
    __syncwarp();
    const int per = (ng + 31) / 32;
    const int g0 = min(ng, lane * per), g1 = min(ng, g0 + per);
    int run = 0;
    for (int g = g0; g < g1; ++g) {
      int rows_g = ctl.goff[g + 1] - ctl.goff[g];
      if (rows_g < 0 || ctl.goff[g + 1] > sg.capacity) {
        record_error(p.err, kErrCapacity);
        rows_g = 0;
      }
      run += ((rows_g + BM - 1) / BM) * sg.n_tiles;
    }
    int incl = run;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      int v = __shfl_up_sync(0xffffffffu, incl, off);
      if (lane >= off) incl += v;
    }
    int excl = incl - run;
    for (int g = g0; g < g1; ++g) {
      ctl.tile_start[g] = excl;
      int rows_g = max(0, ctl.goff[g + 1] - ctl.goff[g]);
      if (ctl.goff[g + 1] > sg.capacity) rows_g = 0;
      excl += ((rows_g + BM - 1) / BM) * sg.n_tiles;
    }
    int total0 = __shfl_sync(0xffffffffu, incl, 31);
    if (lane == 0) {
      ctl.tile_start[ng] = total0;
      ctl.seg0_tiles = total0;
      int total1 = p.nseg > 1 ? ((p.seg[1].rows + BM - 1) / BM) * p.seg[1].n_tiles : 0;
      ctl.total_tiles = total0 + total1;
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = ctl.tmem_base;
  const int total = ctl.total_tiles;

  if (warp == 0) {
    // ---------------- TMA producer
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0;
      int pending_phase[kStages];
      for (int i = 0; i < kStages; ++i) pending_phase[i] = -1;
      bool ok = true;
      for (int tile = blockIdx.x; tile < total && ok; tile += gridDim.x) {
        const TileInfo ti = decode(p, ctl, tile);
        const CUtensorMap* ma = ti.seg == 0 ? &tmA0 : &tmA1;
        const CUtensorMap* mb = ti.seg == 0 ? &tmB0 : &tmB1;
        const int kb_n = p.seg[ti.seg].k_blocks;
        for (int kb = 0; kb < kb_n; ++kb) {
          if (!mbar_wait(smem_u32(&ctl.empty[s]), ph ^ 1u, abort_flag, p.err)) { ok = false; break; }
          const uint32_t fb = smem_u32(&ctl.full[s]);
          mbar_arrive_expect_tx(fb, kABytes + kB8Bytes);
          tma_load_2d(smem_a + s * kABytes, ma, fb, kb * BK, ti.row0);
          tma_load_2d(smem_b8 + s * kB8Bytes, mb, fb, kb * BK, ti.b_row0);
          pending_phase[s] = (int)ph;
          if (++s == kStages) { s = 0; ph ^= 1u; }
        }
      }
      if (!ok)
        for (int i = 0; i < kStages; ++i)
          if (pending_phase[i] >= 0) mbar_drain(smem_u32(&ctl.full[i]), (uint32_t)pending_phase[i]);
    }
  } else if (warp >= 6) {
    // ---------------- e4m3 -> f16 converters (128 threads)
    const int ct = threadIdx.x - 192;
    const int q = ct & 3, rbase = ct >> 2;  // 16 e4m3 bytes of row rbase + 32 i
    int s = 0;
    uint32_t ph = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < total && ok; tile += gridDim.x) {
      const TileInfo ti = decode(p, ctl, tile);
      const int kb_n = p.seg[ti.seg].k_blocks;
      for (int kb = 0; kb < kb_n; ++kb) {
        int wok = 1;
        if (lane == 0) wok = mbar_wait(smem_u32(&ctl.full[s]), ph, abort_flag, p.err) ? 1 : 0;
        wok = __shfl_sync(0xffffffffu, wok, 0);
        if (!wok) { ok = false; break; }
        const uint8_t* src = b8_ptr + s * kB8Bytes;
        uint8_t* dst = b16_ptr + s * kBBytes;
#pragma unroll 2
        for (int i = 0; i < 8; ++i) {
          const int r = rbase + 32 * i;
          const uint4 v = *reinterpret_cast<const uint4*>(src + r * 64 + q * 16);
          const uint32_t w[4] = {v.x, v.y, v.z, v.w};
          uint32_t o[8];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            o[2 * j] = e4m3x2_to_f16x2((uint16_t)(w[j] & 0xFFFFu));
            o[2 * j + 1] = e4m3x2_to_f16x2((uint16_t)(w[j] >> 16));
          }
          // elements 16q .. 16q+15 of row r = 16-byte chunks 2q, 2q+1 of the 128-byte row,
          // placed at chunk ^ (r & 7) (128-byte swizzle)
          const int c0 = (2 * q) ^ (r & 7), c1 = (2 * q + 1) ^ (r & 7);
          *reinterpret_cast<uint4*>(dst + r * 128 + c0 * 16) = make_uint4(o[0], o[1], o[2], o[3]);
          *reinterpret_cast<uint4*>(dst + r * 128 + c1 * 16) = make_uint4(o[4], o[5], o[6], o[7]);
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        mbar_arrive(smem_u32(&ctl.bready[s]));
        if (++s == kStages) { s = 0; ph ^= 1u; }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_f16_f32(BM, BN);
      int s = 0;
      uint32_t ph = 0;
      int it = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < total && ok; tile += gridDim.x, ++it) {
        const TileInfo ti = decode(p, ctl, tile);
        const int acc = it & 1;
        const uint32_t acc_ph = (uint32_t)((it >> 1) & 1);
        if (!mbar_wait(smem_u32(&ctl.tmem_empty[acc]), acc_ph ^ 1u, abort_flag, p.err)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(acc * BN);
        const int kb_n = p.seg[ti.seg].k_blocks;
        for (int kb = 0; kb < kb_n; ++kb) {
          if (!mbar_wait(smem_u32(&ctl.full[s]), ph, abort_flag, p.err) ||
              !mbar_wait(smem_u32(&ctl.bready[s]), ph, abort_flag, p.err)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t adesc = sw128_kmajor_desc(smem_a + s * kABytes);
          const uint64_t bdesc = sw128_kmajor_desc(smem_b + s * kBBytes);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k)
            umma_f16(d_tmem, adesc + (uint64_t)(2 * k), bdesc + (uint64_t)(2 * k), idesc,
                     (kb > 0 || k > 0) ? 1u : 0u);
          umma_commit(smem_u32(&ctl.empty[s]));
          if (++s == kStages) { s = 0; ph ^= 1u; }
        }
        if (!ok) break;
        umma_commit(smem_u32(&ctl.tmem_full[acc]));
      }
      if (!ok) {
        umma_commit(smem_u32(&ctl.mma_done));
        mbar_drain(smem_u32(&ctl.mma_done), 0);
      }
    }
  } else {
    // ---------------- epilogue (warps 2..5)
    const int q = warp & 3;
    const int r_in_tile = q * 32 + lane;
    int it = 0;
    for (int tile = blockIdx.x; tile < total; tile += gridDim.x, ++it) {
      const TileInfo ti = decode(p, ctl, tile);
      const Segment& sg = p.seg[ti.seg];
      const int acc = it & 1;
      const uint32_t acc_ph = (uint32_t)((it >> 1) & 1);
      int ok = 1;
      if (lane == 0) ok = mbar_wait(smem_u32(&ctl.tmem_full[acc]), acc_ph, abort_flag, p.err) ? 1 : 0;
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) break;
      tc_fence_after();
      const uint32_t taddr = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * BN);
      const bool valid = r_in_tile < ti.rows_valid;
      const size_t row = (size_t)(ti.row0 + r_in_tile);
      const float* sc = sg.scale + ti.b_row0;
      if constexpr (EPI == kEpiSwiGLU) {
        __half* crow = reinterpret_cast<__half*>(sg.c) + row * (size_t)sg.ldc;
        const int col0 = ti.n_blk * (BN / 2);
#pragma unroll 1
        for (int c = 0; c < BN / 2; c += 32) {
          // packed columns: 128 gate channels, then the 128 matching up channels
          const int gc = c, uc = c + BN / 2;
          uint32_t g[32], u[32];
          tmem_ld32(taddr + gc, g);
          tmem_ld32(taddr + uc, u);
          tmem_wait_ld();
          uint32_t packed[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const float g0 = __uint_as_float(g[2 * i]) * __ldg(sc + gc + 2 * i);
            const float g1 = __uint_as_float(g[2 * i + 1]) * __ldg(sc + gc + 2 * i + 1);
            const float u0 = __uint_as_float(u[2 * i]) * __ldg(sc + uc + 2 * i);
            const float u1 = __uint_as_float(u[2 * i + 1]) * __ldg(sc + uc + 2 * i + 1);
            packed[i] = pack_f16x2(silu(g0) * u0, silu(g1) * u1);
          }
          const int col = col0 + c;
          if (valid && col < sg.n_store) {
            uint4* dst = reinterpret_cast<uint4*>(crow + col);
#pragma unroll
            for (int v = 0; v < 4; ++v)
              if (col + v * 8 < sg.n_store)
                dst[v] = make_uint4(packed[4 * v], packed[4 * v + 1], packed[4 * v + 2], packed[4 * v + 3]);
          }
        }
      } else {
        const int col0 = ti.n_blk * BN;
#pragma unroll 1
        for (int c = 0; c < BN; c += 32) {
          uint32_t v32[32];
          tmem_ld32(taddr + c, v32);
          tmem_wait_ld();
          uint32_t packed[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            float a0 = __uint_as_float(v32[2 * i]) * __ldg(sc + c + 2 * i);
            float a1 = __uint_as_float(v32[2 * i + 1]) * __ldg(sc + c + 2 * i + 1);
            if constexpr (EPI == kEpiReLU) {
              a0 = fmaxf(a0, 0.0f);
              a1 = fmaxf(a1, 0.0f);
              packed[i] = pack_f16x2(a0, a1);  // ReLU GEMM1 writes the f16 intermediate
            } else {
              packed[i] = pack_bf16x2(a0, a1);  // GEMM2 writes bf16 expert outputs
            }
          }
          const int col = col0 + c;
          if (valid && col < sg.n_store) {
            uint16_t* crow = reinterpret_cast<uint16_t*>(sg.c) + row * (size_t)sg.ldc;
            uint4* dst = reinterpret_cast<uint4*>(crow + col);
#pragma unroll
            for (int v = 0; v < 4; ++v)
              if (col + v * 8 < sg.n_store)
                dst[v] = make_uint4(packed[4 * v], packed[4 * v + 1], packed[4 * v + 2], packed[4 * v + 3]);
          }
        }
      }
      tc_fence_before();
      mbar_arrive(smem_u32(&ctl.tmem_empty[acc]));
    }
  }

  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

}  // namespace gemm8

// ------------------------------------------------------------------ host side
typedef CUresult (*PFN_encodeTiled8)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                     const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                     CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static PFN_encodeTiled8 encode_fn8() {
  static PFN_encodeTiled8 fn = nullptr;
  if (fn == nullptr) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return nullptr;
    fn = reinterpret_cast<PFN_encodeTiled8>(ptr);
  }
  return fn;
}

// f16 activations: [rows, cols], box 128 x 64, 128-byte swizzle.  e4m3 weights: [rows, cols]
// bytes, box 256 x 64, no swizzle (row-major staging for the converters).
static int make_map(CUtensorMap* m, const void* base, uint64_t rows, uint64_t cols, bool fp8) {
  PFN_encodeTiled8 enc = encode_fn8();
  if (enc == nullptr) return DSCA_ERR_CUDA;
  const uint64_t esz = fp8 ? 1 : 2;
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0 || (cols * esz) % 16 != 0) return DSCA_ERR_BAD_ARG;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {cols * esz};
  cuuint32_t box[2] = {64, fp8 ? 256u : 128u};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(m, fp8 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                   const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   fp8 ? CU_TENSOR_MAP_SWIZZLE_NONE : CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? DSCA_OK : DSCA_ERR_CUDA;
}

template <int EPI>
static int launch8(const CUtensorMap& a0, const CUtensorMap& b0, const CUtensorMap& a1, const CUtensorMap& b1,
                   const gemm8::Params& p, int grid, cudaStream_t stream) {
  static PerDeviceOnce attr_once;
  if (attr_once.run([] {
        return cudaFuncSetAttribute(gemm8::grouped_gemm_fp8_kernel<EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    gemm8::kSmemBytes);
      }) != cudaSuccess)
    return DSCA_ERR_CUDA;
  gemm8::grouped_gemm_fp8_kernel<EPI><<<grid, gemm8::kThreads, gemm8::kSmemBytes, stream>>>(a0, b0, a1, b1, p);
  return cudaGetLastError() == cudaSuccess ? DSCA_OK : DSCA_ERR_CUDA;
}

int launch_grouped_ffn_fp8(const dsca_ffn_args* f, int num_sms, cudaStream_t stream) {
  const int grid = f->num_ctas > 0 ? f->num_ctas : num_sms;
  const int segs = f->segments == 0 ? 3 : f->segments;
  const bool shared = f->shared_rows > 0 && (segs & 2);
  const bool routed = (segs & 1) != 0;
  const int phases = f->phases == 0 ? 3 : f->phases;
  if (!routed && !shared) return DSCA_OK;
  const bool glu = f->act == DSCA_ACT_SWIGLU;
  int rc;
  if (phases & 1) {
    CUtensorMap a0, b0, a1, b1;
    if ((rc = make_map(&a0, f->a, (uint64_t)f->capacity, (uint64_t)f->d, false))) return rc;
    if ((rc = make_map(&b0, f->w1, (uint64_t)f->num_experts_w * f->n1p, (uint64_t)f->d, true))) return rc;
    if (shared) {
      if ((rc = make_map(&a1, f->xs, (uint64_t)f->shared_rows, (uint64_t)f->d, false))) return rc;
      if ((rc = make_map(&b1, f->ws1, (uint64_t)f->shared_n1p, (uint64_t)f->d, true))) return rc;
    } else {
      a1 = a0;
      b1 = b0;
    }
    gemm8::Params p{};
    p.epi = glu ? gemm8::kEpiSwiGLU : gemm8::kEpiReLU;
    p.err = f->err;
    p.nseg = shared ? 2 : 1;
    gemm8::Segment& s0 = p.seg[0];
    s0.group_offsets = f->group_offsets;
    s0.group_weight = f->group_weight;
    s0.ngroups = routed ? f->num_groups : 0;
    s0.n_tiles = f->n1p / gemm8::BN;
    s0.b_rows_per_group = f->n1p;
    s0.k_blocks = (f->d + gemm8::BK - 1) / gemm8::BK;
    s0.c = f->h;
    s0.ldc = f->ip;
    s0.n_store = f->ip;
    s0.capacity = f->capacity;
    s0.scale = f->w1_scale;
    if (shared) {
      gemm8::Segment& s1 = p.seg[1];
      s1.ngroups = 1;
      s1.rows = f->shared_rows;
      s1.n_tiles = f->shared_n1p / gemm8::BN;
      s1.b_rows_per_group = f->shared_n1p;
      s1.k_blocks = (f->d + gemm8::BK - 1) / gemm8::BK;
      s1.c = f->hs;
      s1.ldc = f->shared_ip;
      s1.n_store = f->shared_ip;
      s1.capacity = f->shared_rows;
      s1.scale = f->ws1_scale;
    }
    rc = glu ? launch8<gemm8::kEpiSwiGLU>(a0, b0, a1, b1, p, grid, stream)
             : launch8<gemm8::kEpiReLU>(a0, b0, a1, b1, p, grid, stream);
    if (rc) return rc;
  }
  if (phases & 2) {
    CUtensorMap a0, b0, a1, b1;
    if ((rc = make_map(&a0, f->h, (uint64_t)f->capacity, (uint64_t)f->ip, false))) return rc;
    if ((rc = make_map(&b0, f->w2, (uint64_t)f->num_experts_w * f->dp, (uint64_t)f->ip, true))) return rc;
    if (shared) {
      if ((rc = make_map(&a1, f->hs, (uint64_t)f->shared_rows, (uint64_t)f->shared_ip, false))) return rc;
      if ((rc = make_map(&b1, f->ws2, (uint64_t)f->dp, (uint64_t)f->shared_ip, true))) return rc;
    } else {
      a1 = a0;
      b1 = b0;
    }
    gemm8::Params p{};
    p.epi = gemm8::kEpiStore;
    p.err = f->err;
    p.nseg = shared ? 2 : 1;
    gemm8::Segment& s0 = p.seg[0];
    s0.group_offsets = f->group_offsets;
    s0.group_weight = f->group_weight;
    s0.ngroups = routed ? f->num_groups : 0;
    s0.n_tiles = f->dp / gemm8::BN;
    s0.b_rows_per_group = f->dp;
    s0.k_blocks = (f->ip + gemm8::BK - 1) / gemm8::BK;
    s0.c = f->y;
    s0.ldc = f->d;
    s0.n_store = f->d;
    s0.capacity = f->capacity;
    s0.scale = f->w2_scale;
    if (shared) {
      gemm8::Segment& s1 = p.seg[1];
      s1.ngroups = 1;
      s1.rows = f->shared_rows;
      s1.n_tiles = f->dp / gemm8::BN;
      s1.b_rows_per_group = f->dp;
      s1.k_blocks = (f->shared_ip + gemm8::BK - 1) / gemm8::BK;
      s1.c = f->ys;
      s1.ldc = f->d;
      s1.n_store = f->d;
      s1.capacity = f->shared_rows;
      s1.scale = f->ws2_scale;
    }
    if ((rc = launch8<gemm8::kEpiStore>(a0, b0, a1, b1, p, grid, stream))) return rc;
  }
  return DSCA_OK;
}

}  // namespace dsca
