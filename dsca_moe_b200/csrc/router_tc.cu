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
#include "router_select.cuh"

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

// ------------------------------------------------------------------ fused form (d <= 2048)
//
// One kernel from the bf16 rows to the routing outputs.  A cluster of kSplit CTAs takes a
// 128-token tile; CTA r of the cluster owns K steps [r q, (r + 1) q) (q = ceil(ceil(d/128) / 4),
// at most 4 steps of 128) and tokens [32 r, 32 r + 32) of the tile for the selection.
//   1. The W slice planes of the CTA's K steps go to shared memory by TMA (no multicast).  Every
//      thread loads its share of the tile's x rows for those K steps into registers (thread:
//      rows (tid >> 4) + 32 u, u < 4, 16-byte chunk tid & 15 of each step) and reduces the
//      rows' largest exponents over its 16-lane row group; the four CTAs exchange their partial
//      maxima through distributed shared memory, giving every row its exponent R.
//   2. Per K step the threads slice their registers into the three int8 planes: the magnitude
//      F = floor(|v| 2^(147 - R)) is one fma rounded down (|v| 2^(147 - R) + 2^23, the integer
//      part landing in the low mantissa bits; rows with R < 20 pre-scale by 2^64), byte
//      permutes pack the 7-bit slices of four values per word, and negative values negate their
//      bytes ((0x80 - b) ^ 0x80 per byte, selected by the sign mask).  The planes land in the
//      128-byte-swizzled K-major layout of the MMA's A operand (two buffers); one thread issues
//      three int8 MMAs per 32-byte K step, X_j against the stacked planes [W_0; W_1; W_2]
//      (N = 192) into the column window of D_j .. D_j+2 of five zeroed TMEM accumulators,
//      overlapping the slicing of the next step.
//   3. Each CTA combines its accumulators into one exact 64-bit partial per (token, router row)
//      in shared memory; CTA r adds the four partials of its 32 tokens over distributed shared
//      memory, forms the bf16 logits, and runs the selection of router_select.cuh (softmax,
//      top-k, histogram, ranks, fused scan) on them.
// F = floor(|v| 2^(147 - R)) equals the integer form of the C oracle's fixed_row (M << (13 - sh)
// for sh <= 13, M >> (sh - 13) above), so the logits are the same bits as the three-kernel form.
namespace fused {
constexpr int kThreads = router::kThreads;      // 512
constexpr int BM = 128;                         // tokens per tile = TMEM lanes
constexpr int kSplit = 4;                       // CTAs per tile (K ranges)
constexpr int kKStep = 128;                     // K per MMA stage (bytes of each slice plane)
constexpr int kMaxSteps = 4;                    // K steps per CTA
constexpr int kMaxD = kSplit * kMaxSteps * kKStep;  // 2048
constexpr int kWPlane = kRows * kKStep;         // 8 KB: one W plane of one K step
constexpr int kWStage = kSlices * kWPlane;      // 24 KB
constexpr int kXPlane = BM * kKStep;            // 16 KB: one x plane of one K step
constexpr int kXStage = kSlices * kXPlane;      // 48 KB
constexpr int kPartPitch = kRows + 2;           // int64 per staged partial row (bank spread)
constexpr int kSmemBytes = kMaxSteps * kWStage + 2 * kXStage + 1024;
static_assert(kSplit * 32 * kPartPitch * 8 <= 2 * kXStage, "the partial inboxes fit the x slice buffers");
static_assert(kThreads == 16 * 32 && BM * (kKStep / 8) == 4 * kThreads, "four row chunks per thread and step");
}  // namespace fused

__device__ __forceinline__ int ld_dsmem_s32(uint32_t addr, uint32_t rank) {
  int v;
  asm volatile("ld.shared::cluster.u32 %0, [%1];" : "=r"(v) : "r"(mapa_shared(addr, rank)) : "memory");
  return v;
}
__device__ __forceinline__ void st_dsmem_2x64(uint32_t addr, uint32_t rank, long long a, long long b) {
  asm volatile("st.shared::cluster.v2.s64 [%0], {%1, %2};" ::"r"(mapa_shared(addr, rank)), "l"(a), "l"(b) : "memory");
}
__device__ __forceinline__ uint4 ldg_nc_v4(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}
// per byte: the sign of the selected byte replicated (selector nibble bit 3)
__device__ __forceinline__ uint32_t prmt_sign(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t r;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
  return r;
}
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
// 32 lanes x 32 consecutive 32-bit columns of zeros (thread i of the warp writes lane base + i)
__device__ __forceinline__ void tmem_st32_zero(uint32_t taddr) {
  const uint32_t z = 0u;
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,"
      "%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1};" ::"r"(taddr), "r"(z)
      : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t (&r)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
}

// Magnitude bits of one bf16 (bits in the high half of `f32bits`): 2^23 + floor(|v| 2^s) as an
// fp32 bit pattern, so bits [0, 21) hold F.  pre = 2^64 when s > 127 (then scale = 2^(s - 64)).
__device__ __forceinline__ uint32_t fixed_bits(uint32_t f32bits, float pre, float scale) {
  const float v = fabsf(__uint_as_float(f32bits)) * pre;  // exact: a power of two, normal result
  return __float_as_uint(__fmaf_rd(v, scale, 8388608.0f));
}

// Three slice words (plane 0 = F >> 14, plane 1 = (F >> 7) & 127, plane 2 = F & 127, signed)
// of four values with magnitude bits t0..t3 and bf16 words w0 (values 0, 1) and w1 (values 2, 3).
__device__ __forceinline__ void slice4(uint32_t t0, uint32_t t1, uint32_t t2, uint32_t t3, uint32_t w0, uint32_t w1,
                                       uint32_t& p0, uint32_t& p1, uint32_t& p2) {
  const uint32_t lo01 = __byte_perm(t0, t1, 0x5410), lo23 = __byte_perm(t2, t3, 0x5410);  // bits 0..15 of each
  const uint32_t mi01 = __byte_perm(t0, t1, 0x6521), mi23 = __byte_perm(t2, t3, 0x6521);  // bits 8..23 of each
  const uint32_t a2 = __byte_perm(lo01, lo23, 0x6420) & 0x7f7f7f7fu;
  const uint32_t a1 = __byte_perm(lo01 >> 7, lo23 >> 7, 0x6420) & 0x7f7f7f7fu;
  const uint32_t a0 = __byte_perm(mi01 >> 6, mi23 >> 6, 0x6420);  // bits 14..21 (bit 21 is 0)
  const uint32_t m = prmt_sign(w0, w1, 0xFDB9u);                   // 0xff for negative values
  const uint32_t n0 = (0x80808080u - a0) ^ 0x80808080u, n1 = (0x80808080u - a1) ^ 0x80808080u,
                 n2 = (0x80808080u - a2) ^ 0x80808080u;
  p0 = (a0 & ~m) | (n0 & m);
  p1 = (a1 & ~m) | (n1 & m);
  p2 = (a2 & ~m) | (n2 & m);
}

__global__ void __launch_bounds__(fused::kThreads, 1)
    router_fused_kernel(const __grid_constant__ CUtensorMap tmW, const router::Args a, const int32_t* __restrict__ w_exp,
                        int32_t* err) {
  constexpr int BM = fused::BM, kSplit = fused::kSplit, kKStep = fused::kKStep, kMaxSteps = fused::kMaxSteps;
  constexpr int kWPlane = fused::kWPlane, kWStage = fused::kWStage, kXPlane = fused::kXPlane;
  constexpr int kXStage = fused::kXStage, kPartPitch = fused::kPartPitch;
  constexpr int kThreads = fused::kThreads;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  __shared__ uint64_t wfull[kMaxSteps], sfree[2], sliced[2], acc_full, mma_done;
  __shared__ uint32_t tmem_base_s;
  __shared__ int abort_s;
  __shared__ int rpart[BM], rfin[BM], rw_s[kRows];
  __shared__ float lg_s[router::kTokens * router::kLP];
  __shared__ int ids_s[router::kTokens][DSCA_MAX_TOPK];
  __shared__ uint32_t emask[kRows];
  __shared__ int run_s[kRows];
  __shared__ int seg_s[kThreads / kRows][kRows];
  __shared__ int is_last;

  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t w_base = smem_u32(smem);                             // [kMaxSteps][3][64][128]
  uint8_t* xs = smem + kMaxSteps * kWStage;                           // [2][3][128][128]
  const uint32_t x_base = smem_u32(xs);
  const int tid = (int)threadIdx.x, warp = tid >> 5, lane = tid & 31;
  volatile int* abort_flag = &abort_s;
  const uint32_t rank = cluster_ctarank();
  const int row0 = (int)(blockIdx.x / kSplit) * BM;
  const int T = a.T, d = a.d;
  const int nks_total = (d + kKStep - 1) / kKStep;
  const int q = (nks_total + kSplit - 1) / kSplit;
  const int ks0 = min(nks_total, (int)rank * q);
  const int nks = min(nks_total, ks0 + q) - ks0;

  // ---------------- 1. x rows into registers (issued first: the set-up below runs while they
  //                     are in flight), then the rows' exponents
  const int c16 = tid & 15;
  uint4 xv[kMaxSteps][4];
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    const int t = row0 + (tid >> 4) + 32 * u;
#pragma unroll
    for (int s = 0; s < kMaxSteps; ++s) {
      const int k = (ks0 + s) * kKStep + 8 * c16;
      xv[s][u] = (s < nks && t < T && k < d)
                     ? ldg_nc_v4(reinterpret_cast<const uint16_t*>(a.x) + (size_t)t * d + k)
                     : make_uint4(0u, 0u, 0u, 0u);
    }
  }
  if (tid == 0) {
    for (int s = 0; s < kMaxSteps; ++s) mbar_init(smem_u32(&wfull[s]), 1);
    mbar_init(smem_u32(&sfree[0]), 1);
    mbar_init(smem_u32(&sfree[1]), 1);
    mbar_init(smem_u32(&sliced[0]), kThreads);
    mbar_init(smem_u32(&sliced[1]), kThreads);
    mbar_init(smem_u32(&acc_full), 1);
    mbar_init(smem_u32(&mma_done), 1);
    abort_s = 0;
    fence_mbar_init();
  }
  if (tid < kRows) {
    emask[tid] = 0u;
    rw_s[tid] = w_exp[tid];
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(&tmem_base_s), kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = tmem_base_s;

  if (tid == 0) {
    prefetch_tmap(&tmW);
    for (int s = 0; s < nks; ++s) {
      const uint32_t bar = smem_u32(&wfull[s]);
      mbar_arrive_expect_tx(bar, (uint32_t)kWStage);
      const uint32_t dst = w_base + (uint32_t)(s * kWStage);
      for (int j = 0; j < kSlices; ++j)
        tma_load_2d(dst + (uint32_t)(j * kWPlane), &tmW, bar, (ks0 + s) * kKStep, j * kRows);
    }
  }

#pragma unroll
  for (int u = 0; u < 4; ++u) {
    uint32_t m2 = 0u;
#pragma unroll
    for (int s = 0; s < kMaxSteps; ++s) {
      m2 = __vmaxu2(m2, (xv[s][u].x >> 7) & 0x00ff00ffu);
      m2 = __vmaxu2(m2, (xv[s][u].y >> 7) & 0x00ff00ffu);
      m2 = __vmaxu2(m2, (xv[s][u].z >> 7) & 0x00ff00ffu);
      m2 = __vmaxu2(m2, (xv[s][u].w >> 7) & 0x00ff00ffu);
    }
    int r = (int)max(m2 & 0xffffu, m2 >> 16);
    r = max(r, __shfl_xor_sync(0xffffffffu, r, 8));
    r = max(r, __shfl_xor_sync(0xffffffffu, r, 4));
    r = max(r, __shfl_xor_sync(0xffffffffu, r, 2));
    r = max(r, __shfl_xor_sync(0xffffffffu, r, 1));
    if (c16 == 0) rpart[(tid >> 4) + 32 * u] = max(r, 1);
  }
  if (warp < 4) {
    // the five accumulators start at zero (the MMAs below all accumulate): columns [0, 320) of
    // lane quarter `warp`
    const uint32_t z = tmem_base + ((uint32_t)(32 * warp) << 16);
#pragma unroll 1
    for (int c = 0; c < kAcc * kRows; c += 32) tmem_st32_zero(z + (uint32_t)c);
    tmem_wait_st();
    tc_fence_before();
  }
  cluster_sync_all();  // every CTA's partial exponents; the accumulators are zeroed
  if (tid < BM) {
    const uint32_t addr = smem_u32(&rpart[tid]);
    int r = 1;
    for (uint32_t src = 0; src < (uint32_t)kSplit; ++src) r = max(r, ld_dsmem_s32(addr, src));
    rfin[tid] = r;
  }
  __syncthreads();

  // ---------------- 2. slice each K step into the x planes; one thread issues the MMAs
  float pre[4], scl[4];
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    const int sh = 147 - rfin[(tid >> 4) + 32 * u];  // -107 .. 146
    const bool big = sh > 127;
    pre[u] = big ? __uint_as_float((uint32_t)(64 + 127) << 23) : 1.0f;
    scl[u] = __uint_as_float((uint32_t)((big ? sh - 64 : sh) + 127) << 23);
  }
  // every thread slices its share of step s into buffer s & 1 (after the MMAs of step s - 2 have
  // released it) and arrives on sliced[s & 1]; thread 32 waits for the 512 arrivals and the W
  // planes, then issues the step's MMAs (no CTA-wide barrier per step)
  bool issued = false;
#pragma unroll
  for (int s = 0; s < kMaxSteps; ++s) {
    if (s >= nks) break;
    const int b = s & 1;
    if (s >= 2 && !mbar_wait(smem_u32(&sfree[b]), (uint32_t)(((s - 2) >> 1) & 1), abort_flag, err)) break;
    uint8_t* xb = xs + b * kXStage;
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int r = (tid >> 4) + 32 * u;
      const uint4 v = xv[s][u];
      const uint32_t t0 = fixed_bits(v.x << 16, pre[u], scl[u]), t1 = fixed_bits(v.x & 0xffff0000u, pre[u], scl[u]);
      const uint32_t t2 = fixed_bits(v.y << 16, pre[u], scl[u]), t3 = fixed_bits(v.y & 0xffff0000u, pre[u], scl[u]);
      const uint32_t t4 = fixed_bits(v.z << 16, pre[u], scl[u]), t5 = fixed_bits(v.z & 0xffff0000u, pre[u], scl[u]);
      const uint32_t t6 = fixed_bits(v.w << 16, pre[u], scl[u]), t7 = fixed_bits(v.w & 0xffff0000u, pre[u], scl[u]);
      uint32_t p0a, p1a, p2a, p0b, p1b, p2b;
      slice4(t0, t1, t2, t3, v.x, v.y, p0a, p1a, p2a);
      slice4(t4, t5, t6, t7, v.z, v.w, p0b, p1b, p2b);
      // 8 bytes of K at offset 8 c16 of the row, 128-byte swizzle
      const int off = r * kKStep + ((((c16 >> 1) ^ (r & 7))) << 4) + ((c16 & 1) << 3);
      *reinterpret_cast<uint2*>(xb + off) = make_uint2(p0a, p0b);
      *reinterpret_cast<uint2*>(xb + kXPlane + off) = make_uint2(p1a, p1b);
      *reinterpret_cast<uint2*>(xb + 2 * kXPlane + off) = make_uint2(p2a, p2b);
    }
    fence_proxy_async_smem();
    mbar_arrive(smem_u32(&sliced[b]));
    if (tid == 32 && mbar_wait(smem_u32(&sliced[b]), (uint32_t)((s >> 1) & 1), abort_flag, err) &&
        mbar_wait(smem_u32(&wfull[s]), 0u, abort_flag, err)) {
      tc_fence_after();
      // X_j times the three stacked router slice planes [W_0; W_1; W_2] (N = 192) lands on the
      // accumulators D_j | D_j+1 | D_j+2: the three MMAs write overlapping 192-column windows of
      // the 320 zeroed columns D_0 .. D_4 (64 each), so D_s = sum_{j+k=s} X_j W_k
      constexpr uint32_t id192 = idesc_s8_s32(BM, 3 * kRows);
      const uint32_t xa = x_base + (uint32_t)(b * kXStage), wa = w_base + (uint32_t)(s * kWStage);
      const uint64_t x0 = sw128_kmajor_desc(xa), x1 = sw128_kmajor_desc(xa + kXPlane),
                     x2 = sw128_kmajor_desc(xa + 2 * kXPlane);
      const uint64_t w012 = sw128_kmajor_desc(wa);
#pragma unroll
      for (int k = 0; k < kKStep / 32; ++k) {
        const uint64_t o = (uint64_t)(2 * k);  // 32 bytes of K
        umma_i8(tmem_base, x0 + o, w012 + o, id192, 1u);              // D_0 | D_1 | D_2 += X_0 W
        umma_i8(tmem_base + kRows, x1 + o, w012 + o, id192, 1u);      // D_1 | D_2 | D_3 += X_1 W
        umma_i8(tmem_base + 2 * kRows, x2 + o, w012 + o, id192, 1u);  // D_2 | D_3 | D_4 += X_2 W
      }
      umma_commit(smem_u32(&sfree[b]));
      if (s == nks - 1) umma_commit(smem_u32(&acc_full));
      issued = true;
    }
  }
  __syncthreads();
  const bool aborted = abort_s != 0;
  if (aborted) {
    // let issued MMAs and TMA loads finish before the shared memory and TMEM go away
    if (tid == 32 && issued) {
      umma_commit(smem_u32(&mma_done));
      drain(smem_u32(&mma_done), 0);
    }
    if (tid == 0)
      for (int s = 0; s < nks; ++s) drain(smem_u32(&wfull[s]), 0);
    __syncthreads();
  }

  // ---------------- 3. exact 64-bit partials of this CTA's K range, pushed to their owners: the
  // partials of tile rows [32 o, 32 o + 32) go to CTA o's inbox slot [this CTA] (remote stores
  // into its x slice buffers, free once every CTA's MMAs have completed), then each CTA adds the
  // four slots of its own rows from local shared memory
  long long* inbox = reinterpret_cast<long long*>(xs);  // [kSplit][32 rows][kPartPitch]
  long long pvs[2][8];
  {
    const int lq = warp & 3, cg = warp >> 2;  // TMEM lane quarter (tile rows 32 lq + lane); 16 router rows
    bool have = nks > 0 && !aborted;
    if (have) {
      int ok = 1;
      if (lane == 0) ok = mbar_wait(smem_u32(&acc_full), 0u, abort_flag, err) ? 1 : 0;
      have = __shfl_sync(0xffffffffu, ok, 0) != 0;
    }
    if (have) tc_fence_after();
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int e = 16 * cg + 8 * h;
      long long pv[8];
      if (have) {
        const uint32_t ta = tmem_base + ((uint32_t)(32 * lq) << 16) + (uint32_t)e;
        uint32_t d0[8], d1[8], d2[8], d3[8], d4[8];
        tmem_ld8(ta, d0);
        tmem_ld8(ta + kRows, d1);
        tmem_ld8(ta + 2 * kRows, d2);
        tmem_ld8(ta + 3 * kRows, d3);
        tmem_ld8(ta + 4 * kRows, d4);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 8; ++i)
          pv[i] = (long long)(int)d0[i] * (1ll << 28) + (long long)(int)d1[i] * (1ll << 21) +
                  (long long)(int)d2[i] * (1ll << 14) + (long long)(int)d3[i] * (1ll << 7) + (long long)(int)d4[i];
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) pv[i] = 0;
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) pvs[h][i] = pv[i];
    }
  }
  tc_fence_before();
  cluster_sync_all();  // every CTA's MMAs are complete: the inboxes are free
  {
    const int lq = warp & 3, cg = warp >> 2;
    // rows 32 lq + lane belong to CTA lq: slot [rank], row lane
    const uint32_t slot = smem_u32(inbox + ((size_t)rank * 32 + lane) * kPartPitch);
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const uint32_t dst = slot + (uint32_t)(16 * cg + 8 * h) * 8u;
#pragma unroll
      for (int i = 0; i < 8; i += 2) st_dsmem_2x64(dst + 8u * (uint32_t)i, (uint32_t)lq, pvs[h][i], pvs[h][i + 1]);
    }
  }
  cluster_sync_all();  // every CTA's pushes have landed
  {
    // tokens [32 rank, 32 rank + 32) of the tile: 4 router rows per thread, local reads
    const int rl = tid >> 4, eg = 4 * (tid & 15);
    const int tr = 32 * (int)rank + rl;
    long long acc[4] = {0, 0, 0, 0};
#pragma unroll
    for (int src = 0; src < kSplit; ++src) {
      const long long* q = inbox + ((size_t)src * 32 + rl) * kPartPitch + eg;
      const longlong2 a01 = *reinterpret_cast<const longlong2*>(q), a23 = *reinterpret_cast<const longlong2*>(q + 2);
      acc[0] += a01.x;
      acc[1] += a01.y;
      acc[2] += a23.x;
      acc[3] += a23.y;
    }
    const int rx = rfin[tr];
#pragma unroll
    for (int i = 0; i < 4; ++i)
      lg_s[rl * router::kLP + eg + i] = round_bf16(scale_pow2(__ll2float_rn(acc[i]), rx + rw_s[eg + i] - 294));
  }
  __syncthreads();  // lg_s complete (no CTA touches another's shared memory from here on)
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
  const int nblocks = (T + router::kTokens - 1) / router::kTokens;
  router::select_block<__nv_bfloat16>(a, lg_s, ids_s, emask, run_s, seg_s, &is_last, (int)blockIdx.x, nblocks,
                                      (int)gridDim.x);
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

// The fused form: d <= 2048.
static int launch_router_fused(const dsca_router_args* a, cudaStream_t stream) {
  static PerDeviceOnce attr_once;
  const int T = a->T, d16 = (a->d + 15) & ~15;
  CUtensorMap mw;
  int rc;
  if ((rc = make_map_u8(&mw, a->w_slices, (uint64_t)router_tc::kSlices * router_tc::kRows, (uint64_t)d16,
                        router_tc::kRows)))
    return rc;
  auto kern = router_tc::router_fused_kernel;
  if (attr_once.run([&] {
        return cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    router_tc::fused::kSmemBytes);
      }) != cudaSuccess)
    return DSCA_ERR_CUDA;
  router::Args args;
  router::fill_args(a, &args);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(((T + router_tc::fused::BM - 1) / router_tc::fused::BM) * router_tc::fused::kSplit));
  cfg.blockDim = dim3(router_tc::fused::kThreads);
  cfg.dynamicSmemBytes = router_tc::fused::kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = router_tc::fused::kSplit;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, kern, mw, args, a->w_exp, a->err) != cudaSuccess) return DSCA_ERR_CUDA;
  return cudaGetLastError() == cudaSuccess ? DSCA_OK : DSCA_ERR_CUDA;
}

bool router_tc_fused_supported(int d) { return d <= router_tc::fused::kMaxD; }

int launch_router_tc(const dsca_router_args* a, cudaStream_t stream) {
  if (a->d <= router_tc::fused::kMaxD) return launch_router_fused(a, stream);
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
