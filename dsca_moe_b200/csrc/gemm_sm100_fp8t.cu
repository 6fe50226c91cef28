// K5 (fp8-e4m3 expert weights), weights converted into tensor memory.
//
// Same contract as gemm_sm100_fp8.cu (e4m3 weights with one fp32 scale per packed weight row,
// f16 activations, fp32 accumulation, f16 intermediate, bf16 output), computed swap-AB as
// C^T = W . X^T with the converted weights as the A operand of tcgen05.mma read from tensor
// memory: the e4m3 bytes go HBM -> shared memory (TMA) -> registers -> f16 -> tensor memory
// (tcgen05.st), so the converted weights never pass through shared memory again, and the only
// operand the MMA reads from shared memory is the token tile.
//
// Tile: 128 weight rows (TMEM lanes; SwiGLU: the gate and the up rows of 128 channels, two
// slabs) x up to TBN tokens (the MMA N, rounded up to 16) x 64 K per stage.
//   warp 0      TMA producer: the e4m3 weight rows (64-byte rows, 64-byte swizzle) and the f16
//               token rows (128-byte swizzle) of each K step, 8-stage ring.  No multicast.
//   warp 1      TMEM allocator; one thread issues tcgen05.mma kind::f16 with A in tensor memory
//               (M128 N<=TBN K16, four per slab per stage).
//   warps 2-5   epilogue: TMEM lane = weight row, column = token; x the row's scale, SiLU(g) * u
//               (GEMM1) or ReLU or store; each warp stages its 32 x 32 block in shared memory
//               and writes 16-byte pieces of token rows.
//   warps 6-9   converters: thread = weight row; the row's 64 e4m3 bytes of the stage ->
//               cvt.rn.f16x2.e4m3x2 -> tcgen05.st of 32 columns into one of four TMEM slab sets.
// Every wait is bounded (2 s); a timeout records DSCA_ERR_WAIT_TIMEOUT, the producer and the MMA
// thread drain what they issued, TMEM is freed and the kernel returns.
#include <algorithm>

#include "common.cuh"

namespace dsca {
namespace gemm8t {

constexpr int BM = 128;         // weight rows per tile = TMEM lanes
constexpr int BK = 64;          // K per stage
constexpr int kStages = 8;
constexpr int kAStages = 4;     // converted weight slab sets in TMEM
constexpr int kThreads = 320;
constexpr int kTmemCols = 512;
constexpr int kMaxGroups = 256;

enum Epi { kEpiSwiGLU = 0, kEpiReLU = 1, kEpiStore = 2 };

template <int EPI>
struct Cfg {
  static constexpr bool kGlu = EPI == kEpiSwiGLU;
  static constexpr int nA = kGlu ? 2 : 1;           // weight slabs per tile (gate, up)
  static constexpr int TBN = kGlu ? 64 : 128;       // tokens per tile (MMA N at most)
  static constexpr int kW8Bytes = nA * BM * BK;     // e4m3 bytes per stage
  static constexpr int kTBytes = TBN * BK * 2;      // f16 token bytes per stage
  static constexpr int kStageBytes = kW8Bytes + kTBytes;
  static constexpr int kAcc = nA * TBN;             // accumulator columns per tile
  static constexpr int kACols = nA * (BK / 2);      // TMEM columns of one converted slab set
  static constexpr int kAColBase = 2 * kAcc;        // accumulators [2][kAcc], then the slabs
  static constexpr int kStgElems = 32 * 32;
  static constexpr int kSmemBytes = kStages * kStageBytes + 4 * kStgElems * 2 + 1024;
  static_assert(kAColBase + kAStages * kACols <= kTmemCols, "TMEM columns");
};

struct Segment {
  const int32_t* group_offsets;  // device [ngroups + 1], or null = one group of `rows`
  const int32_t* group_weight;   // device [ngroups], or null = identity
  int ngroups, rows;
  int n_blocks;                  // 128-channel weight blocks per group
  int b_rows_per_group;          // packed weight rows per group
  int k_blocks;
  void* c;                       // f16 (GEMM1) or bf16 (GEMM2)
  int ldc, n_store, capacity;
  const float* scale;            // per packed weight row
};

struct Params {
  Segment seg[2];
  int nseg, seg_first;
  int32_t* err;
};

struct TileInfo {
  int seg, row0, rows_valid, w_row0, n_blk;
};

struct SmemCtl {
  uint64_t full[kStages];
  uint64_t empty[kStages];
  uint64_t aready[kAStages];
  uint64_t aempty[kAStages];
  uint64_t tmem_full[2];
  uint64_t tmem_empty[2];
  uint64_t mma_done;
  uint32_t tmem_base;
  int abort_flag;
  int total_tiles, seg0_tiles, seg1_tiles;
  int tile_start[kMaxGroups + 1];
  int goff[kMaxGroups + 1];
  int gw[kMaxGroups];
};

__device__ __forceinline__ void mbar_drain(uint32_t bar, uint32_t parity) {
  const uint64_t t0 = globaltimer_ns();
  while (!mbar_try_wait(bar, parity))
    if (globaltimer_ns() - t0 > kWaitLimitNs) return;
}

__device__ __forceinline__ float silu(float g) { return __fdividef(g, 1.0f + __expf(-g)); }

__device__ __forceinline__ uint32_t e4m3x2_to_f16x2(uint16_t v) {
  uint32_t r;
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(r) : "h"(v));
  return r;
}

__device__ __forceinline__ uint16_t f16_bits(float f) {
  __half h = __float2half_rn(f);
  return *reinterpret_cast<uint16_t*>(&h);
}
__device__ __forceinline__ uint16_t bf16_bits(float f) {
  __nv_bfloat16 h = __float2bfloat16_rn(f);
  return *reinterpret_cast<uint16_t*>(&h);
}

// Instruction descriptor, kind::f16: A = B = f16, D = f32, both K-major.
__host__ __device__ constexpr uint32_t idesc_f16_f32(int M, int N) {
  return (1u << 4) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// D(tmem) (+)= A(tmem) * B(smem desc), kind::f16
__device__ __forceinline__ void umma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// 32 lanes x 32 consecutive 32-bit columns from registers: thread i of the warp writes lane
// (base + i)
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]),
      "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]),
      "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// MMA N for a tile of `ntok` token rows: a multiple of 16, at least 16
__device__ __forceinline__ int tile_n(int ntok) { return max(16, (ntok + 15) & ~15); }

// Tile table (one warp): segment 0 group-major, every group's token tiles x weight blocks.
template <int TBN>
__device__ __forceinline__ void build_table(const Params& p, SmemCtl& ctl, int lane) {
  const Segment& sg = p.seg[0];
  const int ng = sg.ngroups;
  for (int g = lane; g <= ng; g += 32) ctl.goff[g] = sg.group_offsets ? sg.group_offsets[g] : (g == 0 ? 0 : sg.rows);
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
    run += ((rows_g + TBN - 1) / TBN) * sg.n_blocks;
  }
  int incl = run;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const int v = __shfl_up_sync(0xffffffffu, incl, off);
    if (lane >= off) incl += v;
  }
  int excl = incl - run;
  for (int g = g0; g < g1; ++g) {
    ctl.tile_start[g] = excl;
    int rows_g = max(0, ctl.goff[g + 1] - ctl.goff[g]);
    if (ctl.goff[g + 1] > sg.capacity) rows_g = 0;
    excl += ((rows_g + TBN - 1) / TBN) * sg.n_blocks;
  }
  const int total0 = __shfl_sync(0xffffffffu, incl, 31);
  if (lane == 0) {
    ctl.tile_start[ng] = total0;
    ctl.seg0_tiles = total0;
    ctl.seg1_tiles = p.nseg > 1 ? ((p.seg[1].rows + TBN - 1) / TBN) * p.seg[1].n_blocks : 0;
    ctl.total_tiles = total0 + ctl.seg1_tiles;
  }
}

// Tile index of round r for unit u of U (boustrophedon order).
__device__ __forceinline__ int sched_tile(int r, int u, int U) { return r * U + ((r & 1) ? U - 1 - u : u); }

// Weight rows of block n: SwiGLU packs 256-row blocks [128 gate | 128 up] of 128 channels
template <int EPI, int TBN>
__device__ __forceinline__ TileInfo decode(const Params& p, const SmemCtl& s, int tile) {
  constexpr int kBlockRows = EPI == kEpiSwiGLU ? 256 : 128;
  TileInfo ti;
  const int n_first = p.seg_first == 0 ? s.seg0_tiles : s.seg1_tiles;
  int seg, local;
  if (tile < n_first) {
    seg = p.seg_first;
    local = tile;
  } else {
    seg = 1 - p.seg_first;
    local = tile - n_first;
  }
  const Segment& sg = p.seg[seg];
  int row_base, rows, w_base;
  if (seg == 0) {
    int lo = 0, hi = sg.ngroups;
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (s.tile_start[mid] <= local) lo = mid; else hi = mid;
    }
    local -= s.tile_start[lo];
    row_base = s.goff[lo];
    rows = s.goff[lo + 1] - s.goff[lo];
    w_base = s.gw[lo] * sg.b_rows_per_group;
  } else {
    row_base = 0;
    rows = sg.rows;
    w_base = 0;
  }
  const int m_blk = local / sg.n_blocks;
  ti.n_blk = local - m_blk * sg.n_blocks;
  ti.seg = seg;
  ti.row0 = row_base + m_blk * TBN;
  ti.rows_valid = min(TBN, rows - m_blk * TBN);
  ti.w_row0 = w_base + ti.n_blk * kBlockRows;
  return ti;
}

template <int EPI>
__global__ void __launch_bounds__(kThreads, 1)
    fp8_tmem_kernel(const __grid_constant__ CUtensorMap tmW0, const __grid_constant__ CUtensorMap tmT0,
                    const __grid_constant__ CUtensorMap tmW1, const __grid_constant__ CUtensorMap tmT1,
                    const Params p) {
  using C = Cfg<EPI>;
  constexpr int TBN = C::TBN;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  __shared__ SmemCtl ctl;
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  // stage s: e4m3 weight slabs (nA x 128 rows x 64 B), then the f16 token tile (TBN x 128 B)
  const uint32_t smem_stage0 = smem_u32(smem);
  uint16_t* stage_all = reinterpret_cast<uint16_t*>(smem + kStages * C::kStageBytes);

  const int warp = warp_id(), lane = lane_id();
  volatile int* abort_flag = &ctl.abort_flag;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(smem_u32(&ctl.full[s]), 1);
      mbar_init(smem_u32(&ctl.empty[s]), 1);
    }
    for (int a = 0; a < kAStages; ++a) {
      mbar_init(smem_u32(&ctl.aready[a]), 128);
      mbar_init(smem_u32(&ctl.aempty[a]), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(smem_u32(&ctl.tmem_full[a]), 1);
      mbar_init(smem_u32(&ctl.tmem_empty[a]), 4);
    }
    mbar_init(smem_u32(&ctl.mma_done), 1);
    ctl.abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmW0);
    prefetch_tmap(&tmT0);
    if (p.nseg > 1) {
      prefetch_tmap(&tmW1);
      prefetch_tmap(&tmT1);
    }
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(&ctl.tmem_base), kTmemCols);
    tmem_relinquish();
  }
  if (warp == 2) build_table<TBN>(p, ctl, lane);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = ctl.tmem_base;
  const int total = ctl.total_tiles;
  const int unit = (int)blockIdx.x, units = (int)gridDim.x;

  if (warp == 0) {
    // ---------------- TMA producer
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0;
      int pending_phase[kStages];
      for (int i = 0; i < kStages; ++i) pending_phase[i] = -1;
      bool ok = true;
      for (int r = 0; ok; ++r) {
        const int tile = sched_tile(r, unit, units);
        if (tile >= total) break;
        const TileInfo ti = decode<EPI, TBN>(p, ctl, tile);
        const CUtensorMap* mw = ti.seg == 0 ? &tmW0 : &tmW1;
        const CUtensorMap* mt = ti.seg == 0 ? &tmT0 : &tmT1;
        const int kb_n = p.seg[ti.seg].k_blocks;
        for (int kb = 0; kb < kb_n; ++kb) {
          if (!mbar_wait(smem_u32(&ctl.empty[s]), ph ^ 1u, abort_flag, p.err)) { ok = false; break; }
          const uint32_t fb = smem_u32(&ctl.full[s]);
          const uint32_t st = smem_stage0 + (uint32_t)(s * C::kStageBytes);
          mbar_arrive_expect_tx(fb, (uint32_t)C::kStageBytes);
#pragma unroll
          for (int a = 0; a < C::nA; ++a) tma_load_2d(st + (uint32_t)(a * BM * BK), mw, fb, kb * BK, ti.w_row0 + a * BM);
          tma_load_2d(st + (uint32_t)C::kW8Bytes, mt, fb, kb * BK, ti.row0);
          pending_phase[s] = (int)ph;
          if (++s == kStages) { s = 0; ph ^= 1u; }
        }
      }
      if (!ok)
        for (int i = 0; i < kStages; ++i)
          if (pending_phase[i] >= 0) mbar_drain(smem_u32(&ctl.full[i]), (uint32_t)pending_phase[i]);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer
    if (lane == 0) {
      int s = 0, as = 0, it = 0;
      uint32_t ph = 0, aph = 0;
      bool ok = true;
      for (int r = 0; ok; ++r, ++it) {
        const int tile = sched_tile(r, unit, units);
        if (tile >= total) break;
        const TileInfo ti = decode<EPI, TBN>(p, ctl, tile);
        const uint32_t idesc = idesc_f16_f32(BM, tile_n(ti.rows_valid));
        const int acc = it & 1;
        const uint32_t acc_ph = (uint32_t)((it >> 1) & 1);
        if (!mbar_wait(smem_u32(&ctl.tmem_empty[acc]), acc_ph ^ 1u, abort_flag, p.err)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(acc * C::kAcc);
        const int kb_n = p.seg[ti.seg].k_blocks;
        for (int kb = 0; kb < kb_n; ++kb) {
          if (!mbar_wait(smem_u32(&ctl.full[s]), ph, abort_flag, p.err) ||
              !mbar_wait(smem_u32(&ctl.aready[as]), aph, abort_flag, p.err)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t tdesc = sw128_kmajor_desc(smem_stage0 + (uint32_t)(s * C::kStageBytes + C::kW8Bytes));
          const uint32_t a_tmem = tmem_base + (uint32_t)(C::kAColBase + as * C::kACols);
#pragma unroll
          for (int a = 0; a < C::nA; ++a)
#pragma unroll
            for (int k = 0; k < BK / 16; ++k)
              umma_f16_ts(d_tmem + (uint32_t)(a * TBN), a_tmem + (uint32_t)(a * (BK / 2) + 8 * k),
                          tdesc + (uint64_t)(2 * k), idesc, (kb > 0 || k > 0) ? 1u : 0u);
          umma_commit(smem_u32(&ctl.empty[s]));
          umma_commit(smem_u32(&ctl.aempty[as]));
          if (++s == kStages) { s = 0; ph ^= 1u; }
          if (++as == kAStages) { as = 0; aph ^= 1u; }
        }
        if (!ok) break;
        umma_commit(smem_u32(&ctl.tmem_full[acc]));
      }
      if (!ok) {
        umma_commit(smem_u32(&ctl.mma_done));
        mbar_drain(smem_u32(&ctl.mma_done), 0);
      }
    }
  } else if (warp >= 6) {
    // ---------------- converters: thread = weight row 32 q + lane of the tile
    const int q = warp & 3;
    const int row = q * 32 + lane;
    const uint32_t lane_addr = (uint32_t)(q * 32) << 16;
    // 64-byte swizzle of the staged e4m3 rows: 16-byte chunk c of row r sits at c ^ ((r >> 1) & 3)
    const int swz = (row >> 1) & 3;
    int s = 0, as = 0;
    uint32_t ph = 0, aph = 0;
    bool ok = true;
    for (int r = 0; ok; ++r) {
      const int tile = sched_tile(r, unit, units);
      if (tile >= total) break;
      const TileInfo ti = decode<EPI, TBN>(p, ctl, tile);
      const int kb_n = p.seg[ti.seg].k_blocks;
      for (int kb = 0; kb < kb_n; ++kb) {
        int wok = 1;
        if (lane == 0)
          wok = (mbar_wait(smem_u32(&ctl.full[s]), ph, abort_flag, p.err) &&
                 mbar_wait(smem_u32(&ctl.aempty[as]), aph ^ 1u, abort_flag, p.err))
                    ? 1
                    : 0;
        wok = __shfl_sync(0xffffffffu, wok, 0);
        if (!wok) { ok = false; break; }
        tc_fence_after();
        const uint8_t* st = smem + s * C::kStageBytes;
#pragma unroll
        for (int a = 0; a < C::nA; ++a) {
          const uint8_t* src = st + a * BM * BK + row * BK;
          uint32_t v[32];
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            const uint4 u = *reinterpret_cast<const uint4*>(src + ((c ^ swz) * 16));
            const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              v[8 * c + 2 * j] = e4m3x2_to_f16x2((uint16_t)(w[j] & 0xFFFFu));
              v[8 * c + 2 * j + 1] = e4m3x2_to_f16x2((uint16_t)(w[j] >> 16));
            }
          }
          tmem_st32(tmem_base + lane_addr + (uint32_t)(C::kAColBase + as * C::kACols + a * (BK / 2)), v);
        }
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(smem_u32(&ctl.aready[as]));
        if (++s == kStages) { s = 0; ph ^= 1u; }
        if (++as == kAStages) { as = 0; aph ^= 1u; }
      }
    }
  } else {
    // ---------------- epilogue (warps 2..5 -> TMEM lane quarters 2, 3, 0, 1)
    const int q = warp & 3;
    const int wrow = q * 32 + lane;  // the weight row (output channel) this lane holds
    uint16_t* stg = stage_all + (warp - 2) * C::kStgElems;
    int it = 0;
    for (int r = 0;; ++r, ++it) {
      const int tile = sched_tile(r, unit, units);
      if (tile >= total) break;
      const TileInfo ti = decode<EPI, TBN>(p, ctl, tile);
      const Segment& sg = p.seg[ti.seg];
      const int acc = it & 1;
      const uint32_t acc_ph = (uint32_t)((it >> 1) & 1);
      int w_ok = 1;
      if (lane == 0) w_ok = mbar_wait(smem_u32(&ctl.tmem_full[acc]), acc_ph, abort_flag, p.err) ? 1 : 0;
      w_ok = __shfl_sync(0xffffffffu, w_ok, 0);
      if (!w_ok) break;
      tc_fence_after();
      const uint32_t taddr = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * C::kAcc);
      const int ntok = ti.rows_valid;
      const int ncol = tile_n(ntok);
      const float sc0 = __ldg(sg.scale + ti.w_row0 + wrow);
      const float sc1 = C::kGlu ? __ldg(sg.scale + ti.w_row0 + BM + wrow) : 0.0f;
      const int col0 = ti.n_blk * BM + q * 32;  // this warp's 32 output channels
#pragma unroll 1
      for (int c = 0; c < ncol; c += 32) {
        uint32_t v[32];
        tmem_ld32(taddr + (uint32_t)c, v);
        if constexpr (C::kGlu) {
          uint32_t u[32];
          tmem_ld32(taddr + (uint32_t)(TBN + c), u);
          tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 32; ++j)
            stg[j * 32 + lane] = f16_bits(silu(__uint_as_float(v[j]) * sc0) * (__uint_as_float(u[j]) * sc1));
        } else {
          tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const float a = __uint_as_float(v[j]) * sc0;
            if constexpr (EPI == kEpiReLU)
              stg[j * 32 + lane] = f16_bits(fmaxf(a, 0.0f));  // the f16 intermediate
            else
              stg[j * 32 + lane] = bf16_bits(a);  // bf16 expert outputs
          }
        }
        __syncwarp();
#pragma unroll
        for (int rr = 0; rr < 4; ++rr) {
          const int jj = rr * 8 + (lane >> 2), piece = lane & 3;
          const int t = c + jj, col = col0 + piece * 8;
          if (t < ntok && col < sg.n_store) {
            const uint4 val = *reinterpret_cast<const uint4*>(stg + jj * 32 + piece * 8);
            uint16_t* crow = reinterpret_cast<uint16_t*>(sg.c) + (size_t)(ti.row0 + t) * sg.ldc;
            *reinterpret_cast<uint4*>(crow + col) = val;
          }
        }
        __syncwarp();
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&ctl.tmem_empty[acc]));
    }
  }

  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

}  // namespace gemm8t

// ------------------------------------------------------------------ host side
typedef CUresult (*PFN_encodeTiled8t)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                      const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                      CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static PFN_encodeTiled8t encode_fn8t() {
  static PFN_encodeTiled8t fn = nullptr;
  if (fn == nullptr) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return nullptr;
    fn = reinterpret_cast<PFN_encodeTiled8t>(ptr);
  }
  return fn;
}

// e4m3 weights [rows, cols] bytes: box 128 rows x 64 bytes, 64-byte swizzle (the converters read
// one row per thread).  f16 tokens [rows, cols]: box box_rows x 64, 128-byte swizzle (the MMA's
// K-major B operand).
static int make_map_w8(CUtensorMap* m, const void* base, uint64_t rows, uint64_t cols) {
  PFN_encodeTiled8t enc = encode_fn8t();
  if (enc == nullptr) return DSCA_ERR_CUDA;
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0 || cols % 16 != 0) return DSCA_ERR_BAD_ARG;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {cols};
  cuuint32_t box[2] = {64, (cuuint32_t)gemm8t::BM};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? DSCA_OK : DSCA_ERR_CUDA;
}

static int make_map_t16(CUtensorMap* m, const void* base, uint64_t rows, uint64_t cols, uint32_t box_rows) {
  PFN_encodeTiled8t enc = encode_fn8t();
  if (enc == nullptr) return DSCA_ERR_CUDA;
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0 || (cols * 2) % 16 != 0) return DSCA_ERR_BAD_ARG;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {cols * 2};
  cuuint32_t box[2] = {64, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? DSCA_OK : DSCA_ERR_CUDA;
}

template <int EPI>
static int launch8t(const CUtensorMap& w0, const CUtensorMap& t0, const CUtensorMap& w1, const CUtensorMap& t1,
                    const gemm8t::Params& p, int grid, cudaStream_t stream) {
  static PerDeviceOnce attr_once;
  constexpr int smem_bytes = gemm8t::Cfg<EPI>::kSmemBytes;
  if (attr_once.run([] {
        return cudaFuncSetAttribute(gemm8t::fp8_tmem_kernel<EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    smem_bytes);
      }) != cudaSuccess)
    return DSCA_ERR_CUDA;
  gemm8t::fp8_tmem_kernel<EPI><<<grid, gemm8t::kThreads, smem_bytes, stream>>>(w0, t0, w1, t1, p);
  return cudaGetLastError() == cudaSuccess ? DSCA_OK : DSCA_ERR_CUDA;
}

// dsca_grouped_ffn, dtype DSCA_F8E4M3, tile_rows 256: the tensor-memory form above.
int launch_grouped_ffn_fp8_tmem(const dsca_ffn_args* f, int num_sms, cudaStream_t stream) {
  const int grid = f->num_ctas > 0 ? f->num_ctas : num_sms;
  const int segs = f->segments == 0 ? 3 : f->segments;
  const bool shared = f->shared_rows > 0 && (segs & 2);
  const bool routed = (segs & 1) != 0;
  const int phases = f->phases == 0 ? 3 : f->phases;
  if (!routed && !shared) return DSCA_OK;
  const bool glu = f->act == DSCA_ACT_SWIGLU;
  if (f->n1p % 256 != 0 || f->dp % 128 != 0 || f->ip % 128 != 0) return DSCA_ERR_BAD_ARG;
  if (shared && f->shared_ip % 128 != 0) return DSCA_ERR_BAD_ARG;
  int rc;
  if (phases & 1) {
    constexpr uint32_t tg = gemm8t::Cfg<gemm8t::kEpiSwiGLU>::TBN, tr = gemm8t::Cfg<gemm8t::kEpiReLU>::TBN;
    const uint32_t tbn = glu ? tg : tr;
    CUtensorMap w0, t0, w1, t1;
    if ((rc = make_map_w8(&w0, f->w1, (uint64_t)f->num_experts_w * f->n1p, (uint64_t)f->d))) return rc;
    if ((rc = make_map_t16(&t0, f->a, (uint64_t)f->capacity, (uint64_t)f->d, tbn))) return rc;
    if (shared) {
      if ((rc = make_map_w8(&w1, f->ws1, (uint64_t)f->shared_n1p, (uint64_t)f->d))) return rc;
      if ((rc = make_map_t16(&t1, f->xs, (uint64_t)f->shared_rows, (uint64_t)f->d, tbn))) return rc;
    } else {
      w1 = w0;
      t1 = t0;
    }
    gemm8t::Params p{};
    p.err = f->err;
    p.nseg = shared ? 2 : 1;
    p.seg_first = 0;
    gemm8t::Segment& s0 = p.seg[0];
    s0.group_offsets = f->group_offsets;
    s0.group_weight = f->group_weight;
    s0.ngroups = routed ? f->num_groups : 0;
    s0.n_blocks = glu ? f->ip / 128 : f->n1p / 128;
    s0.b_rows_per_group = f->n1p;
    s0.k_blocks = (f->d + gemm8t::BK - 1) / gemm8t::BK;
    s0.c = f->h;
    s0.ldc = f->ip;
    s0.n_store = f->ip;
    s0.capacity = f->capacity;
    s0.scale = f->w1_scale;
    if (shared) {
      gemm8t::Segment& s1 = p.seg[1];
      s1.ngroups = 1;
      s1.rows = f->shared_rows;
      s1.n_blocks = glu ? f->shared_ip / 128 : f->shared_n1p / 128;
      s1.b_rows_per_group = f->shared_n1p;
      s1.k_blocks = (f->d + gemm8t::BK - 1) / gemm8t::BK;
      s1.c = f->hs;
      s1.ldc = f->shared_ip;
      s1.n_store = f->shared_ip;
      s1.capacity = f->shared_rows;
      s1.scale = f->ws1_scale;
    }
    rc = glu ? launch8t<gemm8t::kEpiSwiGLU>(w0, t0, w1, t1, p, grid, stream)
             : launch8t<gemm8t::kEpiReLU>(w0, t0, w1, t1, p, grid, stream);
    if (rc) return rc;
  }
  if (phases & 2) {
    constexpr uint32_t tbn = gemm8t::Cfg<gemm8t::kEpiStore>::TBN;
    CUtensorMap w0, t0, w1, t1;
    if ((rc = make_map_w8(&w0, f->w2, (uint64_t)f->num_experts_w * f->dp, (uint64_t)f->ip))) return rc;
    if ((rc = make_map_t16(&t0, f->h, (uint64_t)f->capacity, (uint64_t)f->ip, tbn))) return rc;
    if (shared) {
      if ((rc = make_map_w8(&w1, f->ws2, (uint64_t)f->dp, (uint64_t)f->shared_ip))) return rc;
      if ((rc = make_map_t16(&t1, f->hs, (uint64_t)f->shared_rows, (uint64_t)f->shared_ip, tbn))) return rc;
    } else {
      w1 = w0;
      t1 = t0;
    }
    gemm8t::Params p{};
    p.err = f->err;
    p.nseg = shared ? 2 : 1;
    p.seg_first = (shared && f->shared_ip > f->ip) ? 1 : 0;  // the longer K first
    gemm8t::Segment& s0 = p.seg[0];
    s0.group_offsets = f->group_offsets;
    s0.group_weight = f->group_weight;
    s0.ngroups = routed ? f->num_groups : 0;
    s0.n_blocks = f->dp / 128;
    s0.b_rows_per_group = f->dp;
    s0.k_blocks = (f->ip + gemm8t::BK - 1) / gemm8t::BK;
    s0.c = f->y;
    s0.ldc = f->d;
    s0.n_store = f->d;
    s0.capacity = f->capacity;
    s0.scale = f->w2_scale;
    if (shared) {
      gemm8t::Segment& s1 = p.seg[1];
      s1.ngroups = 1;
      s1.rows = f->shared_rows;
      s1.n_blocks = f->dp / 128;
      s1.b_rows_per_group = f->dp;
      s1.k_blocks = (f->shared_ip + gemm8t::BK - 1) / gemm8t::BK;
      s1.c = f->ys;
      s1.ldc = f->d;
      s1.n_store = f->d;
      s1.capacity = f->shared_rows;
      s1.scale = f->ws2_scale;
    }
    if ((rc = launch8t<gemm8t::kEpiStore>(w0, t0, w1, t1, p, grid, stream))) return rc;
  }
  return DSCA_OK;
}

}  // namespace dsca
