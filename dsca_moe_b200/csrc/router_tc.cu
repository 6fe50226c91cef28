// K1, tensor-core logits — bf16 router logits by exact fixed-point accumulation on int8 tcgen05
// MMAs, then the selection pass of router.cu (softmax, top-k, histograms, ranks, fused scan).
//
// Arithmetic (the C oracle's oracle_router_logits_fixed): a bf16 value v = s M 2^(e - 134) is
// held relative to the largest exponent R of its row as the 21-bit magnitude
// F = M << (13 - (R - e)) (M >> ((R - e) - 13) once R - e > 13), split into three signed 7-bit
// slices F = a0 2^14 + a1 2^7 + a2.  For a token row X and a router row W the nine slice products
// accumulate exactly in five int32 sums D_s = sum_{j + k = s} X_j . W_k (|D_s| < 3 * 127^2 * d),
// P = sum_s D_s 2^(7 (4 - s)) is formed in 64-bit integers, converted once to fp32 (round to
// nearest), scaled by 2^(R_x + R_w - 294) with IEEE multiplications and rounded to bf16.  P is the
// exact integer dot product of the fixed-point rows, so the logit is the correctly rounded dot
// product whenever no row holds values more than 2^13 below its largest.
//
//   slice_rows_kernel  one warp per row: the row's exponent R, then the three slice planes
//                      ([3][rows][d16] int8, d16 = d rounded up to 16, zero padded)
//   router_mma_kernel  one CTA per 128 tokens: TMA loads the three x slices (128 x 128 bytes each)
//                      and the three router-row slices (64 x 128 bytes) per stage, 3 stages; one
//                      thread issues 9 x 4 tcgen05.mma.kind::i8 (M128 N64 K32) per stage into five
//                      TMEM accumulators (5 x 64 columns); four epilogue warps combine them and
//                      write fp32 logits [T][64] rounded to bf16.  No multicast.  Every wait is
//                      bounded (2 s): a timeout records DSCA_ERR_WAIT_TIMEOUT, drains and frees TMEM.
#include "common.cuh"

namespace dsca {

namespace router_tc {

constexpr int kRows = 64;                              // router rows: E experts, shared gate, zeros
constexpr int BM = 128;                                // tokens per CTA
constexpr int BKB = 128;                               // K bytes (int8 elements) per stage
constexpr int kSlices = 3;
constexpr int kAcc = 5;                                // accumulators D_0 .. D_4
constexpr int kStages = 3;
constexpr int kABytes = BM * BKB;                      // 16 KB per x slice
constexpr int kBBytes = kRows * BKB;                   // 8 KB per router slice
constexpr int kStageBytes = kSlices * (kABytes + kBBytes);
constexpr int kSmemBytes = kStages * kStageBytes + 1024;
constexpr int kThreads = 192;
constexpr int kTmemCols = 512;

// Instruction descriptor, kind::i8: A, B signed int8, D int32, K-major, M x N.
__host__ __device__ constexpr uint32_t idesc_s8_s32(int M, int N) {
  return (2u << 4)                       // D format s32
         | (1u << 7)                     // A signed
         | (1u << 10)                    // B signed
         | ((uint32_t)(N >> 3) << 17)    // N / 8
         | ((uint32_t)(M >> 4) << 24);   // M / 16
}

__device__ __forceinline__ void umma_i8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                        uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Bounded wait that ignores the abort flag (drains in-flight work before exit).
__device__ __forceinline__ void drain(uint32_t bar, uint32_t parity) {
  const uint64_t t0 = globaltimer_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer_ns() - t0 > kWaitLimitNs) return;
  }
}

// f * 2^k by IEEE multiplications, each factor a normal power of two (the oracle's order)
__device__ __forceinline__ float scale_pow2(float f, int k) {
  while (k > 127) {
    f = __fmul_rn(f, __uint_as_float(254u << 23));
    k -= 127;
  }
  while (k < -126) {
    f = __fmul_rn(f, __uint_as_float(1u << 23));
    k += 126;
  }
  return __fmul_rn(f, __uint_as_float((uint32_t)(k + 127) << 23));
}

// 21-bit fixed-point magnitude of one bf16 (bits u) relative to row exponent r, with its sign
__device__ __forceinline__ int fixed_of(uint32_t u, int r) {
  const int b = (int)((u >> 7) & 0xffu), m = (int)(u & 0x7fu);
  const int M = b ? 128 + m : m, e = b ? b : 1, sh = r - e;
  const int f = sh <= 13 ? (M << (13 - sh)) : (sh - 13 < 9 ? (M >> (sh - 13)) : 0);
  return (u & 0x8000u) ? -f : f;
}

__device__ __forceinline__ int row_exp_of(uint32_t u) {
  const int b = (int)((u >> 7) & 0xffu);
  return ((u & 0x7fffu) != 0u) ? max(b, 1) : 1;
}

// one warp per row of `src` ([rows][d] bf16, d % 8 == 0): exponent, then three slice planes
// out[j][row][c] (plane stride plane_rows * d16 bytes), columns d .. d16 zero.  Loads are issued
// kU at a time per lane (independent 16-byte loads in flight), in both passes.
constexpr int kU = 8;
__global__ void __launch_bounds__(256) slice_rows_kernel(const uint16_t* __restrict__ src, int rows, int d, int d16,
                                                          int plane_rows, int8_t* __restrict__ out,
                                                          int32_t* __restrict__ rexp) {
  const int warp = (int)(blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5)), lane = (int)(threadIdx.x & 31);
  if (warp >= plane_rows) return;
  const size_t plane = (size_t)plane_rows * d16;
  int8_t* o = out + (size_t)warp * d16;
  if (warp >= rows) {  // padding rows of the router operand: zeros
    for (int c = lane * 8; c < d16; c += 256)
#pragma unroll
      for (int j = 0; j < kSlices; ++j) *reinterpret_cast<uint2*>(o + j * plane + c) = make_uint2(0u, 0u);
    if (lane == 0) rexp[warp] = 1;
    return;
  }
  const uint16_t* row = src + (size_t)warp * d;
  // pass 1: the row's largest biased exponent (zero and subnormal entries count as 1)
  uint32_t emax2 = 0x00010001u;  // two 16-bit lanes
  for (int base = 0; base < d; base += 256 * kU) {
    uint4 v[kU];
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const int c = base + (u * 32 + lane) * 8;
      v[u] = c < d ? *reinterpret_cast<const uint4*>(row + c) : make_uint4(0u, 0u, 0u, 0u);
    }
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      emax2 = __vmaxu2(emax2, (v[u].x >> 7) & 0x00ff00ffu);
      emax2 = __vmaxu2(emax2, (v[u].y >> 7) & 0x00ff00ffu);
      emax2 = __vmaxu2(emax2, (v[u].z >> 7) & 0x00ff00ffu);
      emax2 = __vmaxu2(emax2, (v[u].w >> 7) & 0x00ff00ffu);
    }
  }
  int r = (int)max(emax2 & 0xffffu, emax2 >> 16);
  r = (int)__reduce_max_sync(0xffffffffu, (unsigned)r);
  // pass 2: slices (the row was just read: these loads hit L1 / L2)
  for (int base = 0; base < d16; base += 256 * kU) {
    uint4 v[kU];
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const int c = base + (u * 32 + lane) * 8;
      v[u] = c < d ? *reinterpret_cast<const uint4*>(row + c) : make_uint4(0u, 0u, 0u, 0u);
    }
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const int c = base + (u * 32 + lane) * 8;
      if (c >= d16) continue;
      const uint32_t w[4] = {v[u].x, v[u].y, v[u].z, v[u].w};
      uint32_t p[kSlices][2] = {{0u, 0u}, {0u, 0u}, {0u, 0u}};
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const uint32_t h = (i & 1) ? (w[i >> 1] >> 16) : (w[i >> 1] & 0xffffu);
        const int f = fixed_of(h, r);
        const int mag = f < 0 ? -f : f;
        const int a[kSlices] = {mag >> 14, (mag >> 7) & 127, mag & 127};
#pragma unroll
        for (int j = 0; j < kSlices; ++j)
          p[j][i >> 2] |= ((uint32_t)(uint8_t)(int8_t)(f < 0 ? -a[j] : a[j])) << (8 * (i & 3));
      }
#pragma unroll
      for (int j = 0; j < kSlices; ++j) *reinterpret_cast<uint2*>(o + j * plane + c) = make_uint2(p[j][0], p[j][1]);
    }
  }
  if (lane == 0) rexp[warp] = r;
}

struct MmaArgs {
  int T, d16;
  const int32_t* x_exp;
  const int32_t* w_exp;
  float* logits;  // [T][64]
  int round_bf16;
  int32_t* err;
};

constexpr int kSplit = 4;                 // CTAs of a cluster share a token tile, each a quarter of K
// TMEM columns (64 per block; the N = 128 MMAs start on multiples of 128): D_0 | D_1, D_2 | D_3,
// E_1 | E_2 (X_1 W_0 and X_1 W_1, added to D_1 and D_2 by the epilogue), D_4
constexpr uint32_t kColD01 = 0, kColD23 = 128, kColE12 = 256, kColD4 = 384;
constexpr int kPitch = kAcc * kRows + 4;  // int32 per staged partial row (padded against bank conflicts)
static_assert(BM * kPitch * 4 <= kStages * kStageBytes, "partials fit the stage buffers");

// 16 consecutive int32 of CTA `rank`'s shared memory (shared::cta address `addr`)
__device__ __forceinline__ void ld_dsmem16(uint32_t addr, uint32_t rank, int32_t (&v)[16]) {
  const uint32_t a = mapa_shared(addr, rank);
#pragma unroll
  for (int q = 0; q < 4; ++q)
    asm volatile("ld.shared::cluster.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v[4 * q]), "=r"(v[4 * q + 1]), "=r"(v[4 * q + 2]), "=r"(v[4 * q + 3])
                 : "r"(a + 16u * q)
                 : "memory");
}

// One cluster of kSplit CTAs per 128-token tile; CTA r of the cluster runs K blocks
// [r q, (r + 1) q) with q = ceil(blocks / kSplit).  Per 32-byte K step: three MMAs against the
// stacked [W_0; W_1] rows (N = 128: X_0 -> D_0 | D_1, X_2 -> D_2 | D_3, X_1 -> E_1 | E_2) and
// three against W_2 (N = 64: X_2 -> D_4, X_0 -> D_2, X_1 -> D_3), six instead of nine.  The
// epilogue stages each CTA's partial sums (D_1 + E_1, D_2 + E_2) in its shared memory; after a
// cluster barrier CTA r adds the kSplit partials of tile rows [32 r, 32 r + 32) (distributed
// shared memory, exact integer sums), forms the logits and writes them.
__global__ void __launch_bounds__(kThreads, 1)
    router_mma_kernel(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmW01,
                      const __grid_constant__ CUtensorMap tmW2, const MmaArgs p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  __shared__ uint64_t full[kStages], empty[kStages], acc_full, mma_done;
  __shared__ uint32_t tmem_base_s;
  __shared__ int abort_s;
  __shared__ int32_t rw_s[kRows];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t smem_a = smem_u32(smem);                              // X_0, X_1, X_2 per stage
  const uint32_t smem_b = smem_a + kStages * kSlices * kABytes;        // [W_0; W_1], W_2 per stage
  int32_t* part = reinterpret_cast<int32_t*>(smem);                     // staged partials (after the MMAs)
  const int warp = warp_id(), lane = lane_id();
  volatile int* abort_flag = &abort_s;
  const uint32_t rank = cluster_ctarank();
  const int row0 = (int)(blockIdx.x / kSplit) * BM;
  const int kb_total = (p.d16 + BKB - 1) / BKB;
  const int kb_per = (kb_total + kSplit - 1) / kSplit;
  const int kb0 = min(kb_total, (int)rank * kb_per);
  const int kb_n = min(kb_total, kb0 + kb_per) - kb0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(smem_u32(&full[s]), 1);
      mbar_init(smem_u32(&empty[s]), 1);
    }
    mbar_init(smem_u32(&acc_full), 1);
    mbar_init(smem_u32(&mma_done), 1);
    abort_s = 0;
    fence_mbar_init();
  }
  if (threadIdx.x < kRows) rw_s[threadIdx.x] = p.w_exp[threadIdx.x];
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmX);
    prefetch_tmap(&tmW01);
    prefetch_tmap(&tmW2);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(&tmem_base_s), kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = tmem_base_s;

  if (warp == 0) {
    // ---------------- TMA producer
    if (lane == 0) {
      int pending[kStages];
      for (int i = 0; i < kStages; ++i) pending[i] = -1;
      int s = 0;
      uint32_t ph = 0;
      bool ok = true;
      for (int kb = 0; kb < kb_n; ++kb) {
        if (!mbar_wait(smem_u32(&empty[s]), ph ^ 1u, abort_flag, p.err)) {
          ok = false;
          break;
        }
        const uint32_t fb = smem_u32(&full[s]);
        const int kx = (kb0 + kb) * BKB;
        mbar_arrive_expect_tx(fb, kStageBytes);
#pragma unroll
        for (int j = 0; j < kSlices; ++j)
          // rows of plane j start at j * T; rows past T read the next plane (or zeros past the
          // last), which only feed accumulator rows that are not stored
          tma_load_2d(smem_a + (uint32_t)((s * kSlices + j) * kABytes), &tmX, fb, kx, j * p.T + row0);
        const uint32_t b = smem_b + (uint32_t)(s * kSlices * kBBytes);
        tma_load_2d(b, &tmW01, fb, kx, 0);                              // W_0 rows, then W_1 rows
        tma_load_2d(b + 2u * kBBytes, &tmW2, fb, kx, 2 * kRows);        // W_2 rows
        pending[s] = (int)ph;
        if (++s == kStages) {
          s = 0;
          ph ^= 1u;
        }
      }
      if (!ok)
        for (int i = 0; i < kStages; ++i)
          if (pending[i] >= 0) drain(smem_u32(&full[i]), (uint32_t)pending[i]);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer
    if (lane == 0 && kb_n > 0) {
      constexpr uint32_t id128 = idesc_s8_s32(BM, 2 * kRows);
      constexpr uint32_t id64 = idesc_s8_s32(BM, kRows);
      int s = 0;
      uint32_t ph = 0;
      bool ok = true;
      for (int kb = 0; kb < kb_n; ++kb) {
        if (!mbar_wait(smem_u32(&full[s]), ph, abort_flag, p.err)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint64_t x0 = sw128_kmajor_desc(smem_a + (uint32_t)((s * kSlices + 0) * kABytes));
        const uint64_t x1 = sw128_kmajor_desc(smem_a + (uint32_t)((s * kSlices + 1) * kABytes));
        const uint64_t x2 = sw128_kmajor_desc(smem_a + (uint32_t)((s * kSlices + 2) * kABytes));
        const uint64_t w01 = sw128_kmajor_desc(smem_b + (uint32_t)(s * kSlices * kBBytes));
        const uint64_t w2 = sw128_kmajor_desc(smem_b + (uint32_t)((s * kSlices + 2) * kBBytes));
#pragma unroll
        for (int k = 0; k < BKB / 32; ++k) {
          const uint64_t o = (uint64_t)(2 * k);  // 32 bytes of K
          const uint32_t acc = (kb > 0 || k > 0) ? 1u : 0u;
          umma_i8(tmem_base + kColD01, x0 + o, w01 + o, id128, acc);    // X_0 W_0 | X_0 W_1
          umma_i8(tmem_base + kColD23, x2 + o, w01 + o, id128, acc);    // X_2 W_0 | X_2 W_1
          umma_i8(tmem_base + kColE12, x1 + o, w01 + o, id128, acc);    // X_1 W_0 | X_1 W_1
          umma_i8(tmem_base + kColD4, x2 + o, w2 + o, id64, acc);       // X_2 W_2
          umma_i8(tmem_base + kColD23, x0 + o, w2 + o, id64, 1u);       // + X_0 W_2 into D_2
          umma_i8(tmem_base + kColD23 + kRows, x1 + o, w2 + o, id64, 1u);  // + X_1 W_2 into D_3
        }
        umma_commit(smem_u32(&empty[s]));
        if (++s == kStages) {
          s = 0;
          ph ^= 1u;
        }
      }
      if (ok) {
        umma_commit(smem_u32(&acc_full));
      } else {
        umma_commit(smem_u32(&mma_done));
        drain(smem_u32(&mma_done), 0);
      }
    }
  } else {
    // ---------------- stage this CTA's partial sums: warps 2..5 -> TMEM lane quarters 2, 3, 0, 1
    const int q = warp & 3;
    int w_ok = 1;
    if (kb_n > 0) {
      if (lane == 0) w_ok = mbar_wait(smem_u32(&acc_full), 0u, abort_flag, p.err) ? 1 : 0;
      w_ok = __shfl_sync(0xffffffffu, w_ok, 0);
    }
    int32_t* dst = part + (size_t)(q * 32 + lane) * kPitch;
    if (kb_n > 0 && w_ok) {
      tc_fence_after();
      const uint32_t taddr = tmem_base + ((uint32_t)(q * 32) << 16);
      // staged D_s (s = 0..4) at columns 64 s of the row; D_1 and D_2 add the E blocks
#pragma unroll 1
      for (int c = 0; c < kAcc * kRows; c += 32) {
        const int sidx = c / kRows, off = c % kRows;
        const uint32_t col = sidx == 4 ? kColD4 + (uint32_t)off : (uint32_t)c;  // D_0..D_3 are contiguous
        uint32_t v[32];
        tmem_ld32(taddr + col, v);
        tmem_wait_ld();
        if (sidx == 1 || sidx == 2) {
          uint32_t e[32];
          tmem_ld32(taddr + kColE12 + (uint32_t)((sidx - 1) * kRows + off), e);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = (uint32_t)((int32_t)v[i] + (int32_t)e[i]);
        }
#pragma unroll
        for (int i = 0; i < 32; i += 4)
          *reinterpret_cast<int4*>(dst + c + i) = make_int4((int)v[i], (int)v[i + 1], (int)v[i + 2], (int)v[i + 3]);
      }
    } else {
      for (int c = 0; c < kAcc * kRows; c += 4) *reinterpret_cast<int4*>(dst + c) = make_int4(0, 0, 0, 0);
    }
    tc_fence_before();
  }
  cluster_sync_all();  // every CTA of the cluster has staged its partials
  if (warp >= 2) {
    // ---------------- rows [32 rank, 32 rank + 32) of the tile: add the kSplit partials
    const int et = (int)threadIdx.x - 64;       // 0..127
    const int rl = 32 * (int)rank + (et >> 2);  // tile row
    const int cg = (et & 3) * 16;               // 16 router rows
    const int t = row0 + rl;
    long long acc[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) acc[i] = 0;
#pragma unroll 1
    for (int sidx = 0; sidx < kAcc; ++sidx) {
      int32_t sum[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) sum[i] = 0;
      const uint32_t a = smem_u32(part + (size_t)rl * kPitch + sidx * kRows + cg);
#pragma unroll 1
      for (uint32_t src = 0; src < (uint32_t)kSplit; ++src) {
        int32_t v[16];
        ld_dsmem16(a, src, v);
#pragma unroll
        for (int i = 0; i < 16; ++i) sum[i] += v[i];
      }
#pragma unroll
      for (int i = 0; i < 16; ++i) acc[i] = acc[i] * 128 + (long long)sum[i];
    }
    if (t < p.T) {
      const int rx = p.x_exp[t];
      float4* out = reinterpret_cast<float4*>(p.logits + (size_t)t * kRows + cg);
#pragma unroll
      for (int i = 0; i < 16; i += 4) {
        float f[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const float l = scale_pow2(__ll2float_rn(acc[i + u]), rx + rw_s[cg + i + u] - 294);
          f[u] = p.round_bf16 ? round_bf16(l) : l;
        }
        out[i / 4] = make_float4(f[0], f[1], f[2], f[3]);
      }
    }
  }
  cluster_sync_all();  // the peers have read this CTA's partials
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

}  // namespace router_tc

int launch_router(const dsca_router_args* p, cudaStream_t stream, const float* logits_in);

// 2-D uint8 tensor map over a row-major [rows, cols] byte matrix, box = box_rows x 128 bytes,
// 128-byte swizzle (the K-major layout tcgen05 reads).
static int make_map_u8(CUtensorMap* m, const void* base, uint64_t rows, uint64_t cols, uint32_t box_rows) {
  typedef CUresult (*Encode)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                             const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                             CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
  static Encode enc = nullptr;
  if (enc == nullptr) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return DSCA_ERR_CUDA;
    enc = reinterpret_cast<Encode>(fn);
  }
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0 || cols % 16 != 0) return DSCA_ERR_BAD_ARG;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {cols};
  cuuint32_t box[2] = {128, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? DSCA_OK : DSCA_ERR_CUDA;
}

// Router rows [R][d] bf16 -> slice planes [3][64][d16] and exponents [64] (rows R..63 zero).
int launch_router_pack_i8(const void* rows, int R, int d, void* slices, int32_t* exps, cudaStream_t stream) {
  const int d16 = (d + 15) & ~15;
  router_tc::slice_rows_kernel<<<(router_tc::kRows + 7) / 8, 256, 0, stream>>>(
      reinterpret_cast<const uint16_t*>(rows), R, d, d16, router_tc::kRows, reinterpret_cast<int8_t*>(slices), exps);
  return cudaGetLastError() == cudaSuccess ? DSCA_OK : DSCA_ERR_CUDA;
}

int launch_router_tc(const dsca_router_args* a, cudaStream_t stream) {
  static PerDeviceOnce attr_once;
  const int T = a->T, d16 = (a->d + 15) & ~15;
  router_tc::slice_rows_kernel<<<(T + 7) / 8, 256, 0, stream>>>(reinterpret_cast<const uint16_t*>(a->x), T, a->d,
                                                                 d16, T, reinterpret_cast<int8_t*>(a->x_slices),
                                                                 a->x_exp);
  if (cudaGetLastError() != cudaSuccess) return DSCA_ERR_CUDA;
  CUtensorMap mx, mw01, mw2;
  int rc;
  const uint64_t wrows = (uint64_t)router_tc::kSlices * router_tc::kRows;
  if ((rc = make_map_u8(&mx, a->x_slices, (uint64_t)router_tc::kSlices * T, (uint64_t)d16, router_tc::BM))) return rc;
  if ((rc = make_map_u8(&mw01, a->w_slices, wrows, (uint64_t)d16, 2 * router_tc::kRows))) return rc;
  if ((rc = make_map_u8(&mw2, a->w_slices, wrows, (uint64_t)d16, router_tc::kRows))) return rc;
  auto kern = router_tc::router_mma_kernel;
  if (attr_once.run([&] {
        return cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, router_tc::kSmemBytes);
      }) != cudaSuccess)
    return DSCA_ERR_CUDA;
  router_tc::MmaArgs p;
  p.T = T;
  p.d16 = d16;
  p.x_exp = a->x_exp;
  p.w_exp = a->w_exp;
  p.logits = a->logits_f32;
  p.round_bf16 = 1;
  p.err = a->err;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(((T + router_tc::BM - 1) / router_tc::BM) * router_tc::kSplit));
  cfg.blockDim = dim3(router_tc::kThreads);
  cfg.dynamicSmemBytes = router_tc::kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = router_tc::kSplit;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, kern, mx, mw01, mw2, p) != cudaSuccess) return DSCA_ERR_CUDA;
  if (cudaGetLastError() != cudaSuccess) return DSCA_ERR_CUDA;
  return launch_router(a, stream, a->logits_f32);
}

}  // namespace dsca
