// Declarations shared by the two tcgen05 grouped-GEMM kernels (single-CTA tiles in
// gemm_sm100.cu, CTA-pair swap-AB tiles in gemm_sm100_pair.cu): segments, tile decoding, the
// per-CTA control block and the device-side group table.
#pragma once

#include "common.cuh"
#include "ep.cuh"

namespace dsca {
namespace gemm {

constexpr int BN = 256, BK = 64;
constexpr int kThreads = 192;
constexpr int kTmemCols = 512;
constexpr int kMaxGroups = 256;
constexpr int kMaxStages = 6;

// kEpiSwiGLU2: SwiGLU on CTA pairs with the gate and the up rows of a CTA's 64 channels as one
// 128-row M operand (one accumulator; the gate and up halves meet in shared memory)
enum Epi { kEpiSwiGLU = 0, kEpiReLU = 1, kEpiStore = 2, kEpiSwiGLU2 = 3 };

// One GEMM segment: the routed experts (row groups with device-side offsets) or the shared
// expert (one group over all tokens).  "b" is the weight operand: [groups * b_rows_per_group, K].
struct Segment {
  const int32_t* group_offsets;  // device [ngroups + 1], or null = one group of `rows`
  const int32_t* group_weight;   // device [ngroups], or null = identity
  const int32_t* group_order;    // device [ngroups]: execution position -> group, or null = identity
  int ngroups;
  int rows;
  int n_tiles;                   // 256-wide blocks of weight rows per group
  int n_full;                    // hybrid tiles (Params::hybrid): 128-channel blocks per full tile
  int b_rows_per_group;
  int k_blocks;
  __nv_bfloat16* c;
  int ldc;
  int n_store;
  int capacity;
  // expert parallel: when set, output row r of group e belongs to chunk (src, e) of the
  // receive buffer and is stored straight into rank src's return buffer (peer memory)
  const ep::Ctx* ep;
  // fp8-e4m3 weights with two-term e4m3 tokens (pair kernel, F8): the lo plane's first byte
  // column in a token row, 1 / s per token row, and the scale per packed weight row
  int t_lo;
  const float* t_scale;
  const float* w_scale;
  // tile order inside a group: 0 = the weight blocks of one token block after another (token
  // block major); 1 = the token blocks of one weight block after another (weight block major:
  // a weight block is read by all its token blocks back to back, while it is in L2)
  int wmajor;
};

struct Params {
  Segment seg[2];
  int nseg;
  int seg_first;  // segment whose tiles come first
  int epi;
  int32_t* err;
  ep::Ctx* ep_signal;  // set: signal the return flag at every peer once the grid is done
  // launched as a programmatic dependent of the kernel that writes segment 0's A rows: the
  // producer runs griddepcontrol.wait before its first segment-0 load
  int pdl_seg0_wait;
  // launched as a programmatic dependent of the kernel that writes both segments' A rows (GEMM2
  // after GEMM1): the producer runs griddepcontrol.wait before its first load
  int pdl_wait_all;
  // two segments: -1 = all of seg_first's tiles, then the other segment's; >= 0 = this many of
  // seg_first's tiles first, then the two segments' remaining tiles interleaved in proportion
  // to their counts, so that at any time some SMs run the routed experts' tiles (which stream
  // every expert's weights from HBM) while the others run the shared expert's (tensor bound)
  int interleave_lead;
  // L2 policies of the loads: 0 = default; 1 = routed experts' weights (segment 0, streamed from
  // DRAM and mostly read once) evict-first, shared-expert weights and token rows evict-last
  int l2_hints;
  // routed tiles (segment 0): the producer prefetches into L2 the operand boxes this many K
  // blocks ahead of its shared-memory loads (0 = off), so that a tile whose expert weights are
  // not yet in L2 has more DRAM reads in flight than its shared-memory stages hold
  int l2_ahead;
  // CTA-pair SwiGLU GEMM1 only: every whole 256-token block of a group is one non-swapped tile
  // (tokens as M = 256 over the pair, 128 channels' gate and up rows as N = 256, Segment::n_full
  // blocks), the remaining < 256 tokens swap-AB tiles as usual
  int hybrid;
  // dynamic tile schedule: [0] the launch's tile ticket counter, [1] its exit counter (both zero
  // at launch; the last CTA to exit zeroes them), or null = the static boustrophedon schedule
  uint32_t* tile_counter;
  // shared-expert handoff (dsca_ffn_args::shared_handoff): GEMM1 counts its epilogue warps'
  // finished shared-expert tiles in seg1_done[0] and sets seg1_done[1] when all are stored;
  // GEMM2 starts its shared-expert tiles once seg1_flag[0] is set (and zeroes both words when
  // its last CTA exits).  Null = off.
  uint32_t* seg1_done;
  uint32_t* seg1_flag;
};

// A tile: token rows [row0, row0 + rows_valid) of group `group`, weight rows [b_row0, b_row0 + 256)
// (weight block n_blk of the group).
struct TileInfo {
  int seg, group, row0, rows_valid, b_row0, n_blk;
  int full;  // hybrid: a non-swapped 256-token tile (b_row0 = its 256-row [gate | up] block)
};

// Tiles of a group of `rows` token rows: ceil(rows / TBM) row tiles x n_tiles weight blocks, or
// with hybrid tiles floor(rows / 256) x n_full full tiles plus the remainder's row tiles.
template <int TBM>
__device__ __forceinline__ int group_tiles(int rows, const Segment& sg, int hybrid) {
  if (!hybrid) return ((rows + TBM - 1) / TBM) * sg.n_tiles;
  const int full = rows / 256, rest = rows - 256 * full;
  return full * sg.n_full + ((rest + TBM - 1) / TBM) * sg.n_tiles;
}

// Tile `l` of a group (rows rows starting at row_base, weights starting at weight row w_base).
template <int TBM>
__device__ __forceinline__ void decode_in_group(TileInfo& ti, int l, int rows, int row_base, int w_base,
                                                const Segment& sg, int hybrid) {
  const int full = hybrid ? rows / 256 : 0;
  const int nf = full * sg.n_full;
  if (l < nf) {
    const int m_blk = l / sg.n_full;
    ti.n_blk = l - m_blk * sg.n_full;
    ti.full = 1;
    ti.row0 = row_base + 256 * m_blk;
    ti.rows_valid = 256;
    ti.b_row0 = w_base + ti.n_blk * BN;
    return;
  }
  l -= nf;
  int m_blk;
  if (sg.wmajor) {
    const int nm = max(1, (rows - 256 * full + TBM - 1) / TBM);
    ti.n_blk = l / nm;
    m_blk = l - ti.n_blk * nm;
  } else {
    m_blk = l / sg.n_tiles;
    ti.n_blk = l - m_blk * sg.n_tiles;
  }
  ti.full = 0;
  ti.row0 = row_base + 256 * full + m_blk * TBM;
  ti.rows_valid = min(TBM, rows - 256 * full - m_blk * TBM);
  ti.b_row0 = w_base + ti.n_blk * BN;
}

// Destination row pointer of a routed output row in the expert-parallel return path.
__device__ __forceinline__ __nv_bfloat16* ep_return_row(const ep::Ctx* c, int e, int r, int ldc) {
  for (int src = 0; src < c->G; ++src) {
    const int cs = c->chunk_start[e][src];
    if (r >= cs && r < cs + c->chunk_len[e][src])
      return reinterpret_cast<__nv_bfloat16*>(c->ret[src]) + (size_t)(c->ret_start[e][src] + r - cs) * ldc;
  }
  return nullptr;
}

// dsca_ffn_args::tile_order bits 1 and 2: weight-block-major order for the shared expert's
// segment (1) and the routed groups (0)
inline void set_weight_major(Params& p, int tile_order) {
  p.seg[0].wmajor = (tile_order >> 2) & 1;
  p.seg[1].wmajor = (tile_order >> 1) & 1;
}

constexpr int kTQ = 4;  // tile queue depth (tiles the producer may run ahead of the consumers)

struct SmemCtl {
  uint64_t tq_full[kTQ];   // tile id of round r published (1 arrival: the tile source)
  uint64_t tq_empty[kTQ];  // read by every consumer of the CTA (count set by the kernel)
  int tq[kTQ];
  uint64_t full[kMaxStages];
  uint64_t empty[kMaxStages];
  uint64_t tmem_full[2];
  uint64_t tmem_empty[2];
  uint64_t mma_done;
  uint64_t xfull[2][2][2];   // kEpiSwiGLU2: exchange half [warp pair][buffer][sender] written
  uint64_t xempty[2][2][2];  // ... and read by the other warp
  uint32_t tmem_base;
  int abort_flag;
  int total_tiles;
  int seg0_tiles;
  int seg1_tiles;
  int tile_start[kMaxGroups + 1];  // segment 0: prefix of tiles per execution position
  int goff[kMaxGroups + 1];
  int gw[kMaxGroups];
  int gord[kMaxGroups];            // execution position -> group
};

// Tile schedule.  The segment with the longer K (p.seg_first) comes first, then the other; inside
// segment 0 tiles are group-major (a group's M tiles, then its N blocks), so the tiles that
// read one expert's weights run close together and hit L2.  Unit u of U takes tiles in
// boustrophedon order (round r: r U + u for even r, r U + U - 1 - u for odd r), which evens out
// the per-unit work when one segment's tiles are longer.  Built by one warp from the device-side
// group offsets (no host sync).
template <int TBM>
__device__ __forceinline__ void build_group_table(const Params& p, SmemCtl& ctl, int lane) {
  const Segment& sg = p.seg[0];
  const int ng = sg.ngroups;
  for (int g = lane; g <= ng; g += 32)
    ctl.goff[g] = sg.group_offsets ? sg.group_offsets[g] : (g == 0 ? 0 : sg.rows);
  for (int g = lane; g < ng; g += 32) ctl.gw[g] = sg.group_weight ? sg.group_weight[g] : g;
  for (int i = lane; i < ng; i += 32) {
    int g = sg.group_order ? sg.group_order[i] : i;
    if (g < 0 || g >= ng) {
      record_error(p.err, kErrIndex);
      g = i;
    }
    ctl.gord[i] = g;
  }
  __syncwarp();
  // each lane scans a contiguous run of execution positions, then a warp scan stitches the runs
  const int per = (ng + 31) / 32;
  const int g0 = min(ng, lane * per), g1 = min(ng, g0 + per);
  int run = 0;
  for (int i = g0; i < g1; ++i) {
    const int g = ctl.gord[i];
    int rows_g = ctl.goff[g + 1] - ctl.goff[g];
    if (rows_g < 0 || ctl.goff[g + 1] > sg.capacity) {
      record_error(p.err, kErrCapacity);
      rows_g = 0;
    }
    run += group_tiles<TBM>(rows_g, sg, p.hybrid);
  }
  int incl = run;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    int v = __shfl_up_sync(0xffffffffu, incl, off);
    if (lane >= off) incl += v;
  }
  int excl = incl - run;
  for (int i = g0; i < g1; ++i) {
    const int g = ctl.gord[i];
    ctl.tile_start[i] = excl;
    int rows_g = max(0, ctl.goff[g + 1] - ctl.goff[g]);
    if (ctl.goff[g + 1] > sg.capacity) rows_g = 0;
    excl += group_tiles<TBM>(rows_g, sg, p.hybrid);
  }
  int total0 = __shfl_sync(0xffffffffu, incl, 31);
  if (lane == 0) {
    ctl.tile_start[ng] = total0;
    ctl.seg0_tiles = total0;
    int total1 = 0;
    if (p.nseg > 1) total1 = group_tiles<TBM>(p.seg[1].rows, p.seg[1], p.hybrid);
    ctl.seg1_tiles = total1;
    ctl.total_tiles = total0 + total1;
  }
}

// Tile index of round r for unit u of U (boustrophedon order).
__device__ __forceinline__ int sched_tile(int r, int u, int U) { return r * U + ((r & 1) ? U - 1 - u : u); }

// The tile of round r, from the launch's ticket counter (Params::tile_counter: every unit takes
// the next tile when it is ready for one, so long and short tiles spread by their actual
// durations) or the static schedule; `total` or more past the last tile.
__device__ __forceinline__ int ticket_tile(const Params& p, int r, int u, int U) {
  return p.tile_counter != nullptr ? (int)atomicAdd(p.tile_counter, 1u) : sched_tile(r, u, U);
}

// Tile queue, consumer side (one thread): the tile of round r, or -1 past the last tile or when
// the wait ran out (the abort flag is then set).  Arrives on tq_empty[slot] once the id is read:
// this CTA's barrier, or with kCluster the barrier at shared::cluster address empty_bars[slot]
// (the even CTA's of a pair).
template <bool kCluster>
__device__ __forceinline__ int tq_take(SmemCtl& ctl, int r, volatile int* abort_flag, int32_t* err,
                                       const uint32_t* empty_bars) {
  const int slot = r % kTQ;
  if (!mbar_wait<kCluster>(smem_u32(&ctl.tq_full[slot]), (uint32_t)((r / kTQ) & 1), abort_flag, err)) return -1;
  const int tile = *reinterpret_cast<volatile int*>(&ctl.tq[slot]);
  if constexpr (kCluster) mbar_arrive_remote(empty_bars[slot]);
  else mbar_arrive(smem_u32(&ctl.tq_empty[slot]));
  return tile;
}

// The last CTA to exit zeroes the launch's counters (every other CTA has drawn its last ticket),
// and, in GEMM2, the shared-expert handoff words (every GEMM2 CTA waited for GEMM1's completion
// before exiting, and GEMM1 touches them no more once the flag is set).
__device__ __forceinline__ void tile_counter_exit(const Params& p) {
  if (p.tile_counter == nullptr) return;
  __threadfence();
  if (atomicAdd(p.tile_counter + 1, 1u) == gridDim.x - 1u) {
    p.tile_counter[0] = 0u;
    p.tile_counter[1] = 0u;
    if (p.seg1_flag != nullptr) {
      p.seg1_flag[-1] = 0u;
      p.seg1_flag[0] = 0u;
    }
    __threadfence();
  }
}

// GEMM1 epilogue warp, after storing its part of a shared-expert tile: count it; the warp that
// completes the count (warps_per_tile x the segment's tiles) raises the flag.  Every lane fences
// its own stores before the warp's count.
__device__ __forceinline__ void seg1_tile_stored(const Params& p, const SmemCtl& s, int lane,
                                                 unsigned warps_per_tile) {
  __threadfence();
  __syncwarp();
  if (lane == 0) {
    const unsigned old = atomicAdd(p.seg1_done, 1u);
    if (old + 1u == warps_per_tile * (unsigned)s.seg1_tiles) {
      __threadfence();
      atomicExch(p.seg1_done + 1, 1u);
    }
  }
}

// GEMM2 producer: bounded wait for the shared-expert handoff flag, then make GEMM1's stores
// visible to this thread's bulk-tensor (async proxy) loads.
__device__ __forceinline__ bool wait_seg1_flag(const Params& p, volatile int* abort_flag) {
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t it = 0;; ++it) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p.seg1_flag) : "memory");
    if (v != 0u) break;
    if (*abort_flag) return false;
    if (globaltimer_ns() - t0 > kWaitLimitNs) {
      record_error(p.err, kErrWaitTimeout);
      *abort_flag = 1;
      return false;
    }
    __nanosleep(200);
  }
  asm volatile("fence.proxy.async.global;" ::: "memory");
  return true;
}

template <int TBM>
__device__ __forceinline__ TileInfo decode(const Params& p, const SmemCtl& s, int tile) {
  TileInfo ti;
  const int n_first = p.seg_first == 0 ? s.seg0_tiles : s.seg1_tiles;
  const int n_second = s.seg0_tiles + s.seg1_tiles - n_first;
  int seg, local;
  const int lead = min(p.interleave_lead, n_first);
  if (p.interleave_lead < 0 || n_second == 0 || tile < lead) {
    if (tile < n_first) {
      seg = p.seg_first;
      local = tile;
    } else {
      seg = 1 - p.seg_first;
      local = tile - n_first;
    }
  } else {
    // position i of the interleaved rest: c(i) = floor(i * n_second / rest) of the first i
    // positions belong to the second segment; position i is the second segment's c(i)-th tile
    // when c(i + 1) > c(i), else the first segment's (lead + i - c(i))-th
    const long long i = tile - lead, rest = (long long)(n_first - lead) + n_second;
    const int c0 = (int)(i * n_second / rest), c1 = (int)((i + 1) * n_second / rest);
    if (c1 > c0) {
      seg = 1 - p.seg_first;
      local = c0;
    } else {
      seg = p.seg_first;
      local = lead + (int)i - c0;
    }
  }
  if (seg == 0) {
    const Segment& sg = p.seg[0];
    int lo = 0, hi = sg.ngroups;  // g with tile_start[g] <= local < tile_start[g + 1]
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (s.tile_start[mid] <= local) lo = mid; else hi = mid;
    }
    const int g = s.gord[lo];
    ti.seg = 0;
    ti.group = g;
    decode_in_group<TBM>(ti, local - s.tile_start[lo], s.goff[g + 1] - s.goff[g], s.goff[g],
                         s.gw[g] * sg.b_rows_per_group, sg, p.hybrid);
  } else {
    ti.seg = 1;
    ti.group = 0;
    decode_in_group<TBM>(ti, local, p.seg[1].rows, 0, 0, p.seg[1], p.hybrid);
  }
  return ti;
}

// Bounded wait that ignores the abort flag (used to drain in-flight work before exit).
__device__ __forceinline__ void mbar_drain(uint32_t bar, uint32_t parity) {
  const uint64_t t0 = globaltimer_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer_ns() - t0 > kWaitLimitNs) return;
  }
}

// SiLU for the epilogues (bf16 outputs): fast exponential and division
__device__ __forceinline__ float silu(float g) { return __fdividef(g, 1.0f + __expf(-g)); }

}  // namespace gemm

// 2-D bf16 tensor map over a row-major [rows, cols] matrix, box = box_rows x 64, 128B swizzle.
int make_map_bf16(CUtensorMap* m, const void* base, uint64_t rows, uint64_t cols, uint32_t box_rows);
// The CTA-pair swap-AB path of dsca_grouped_ffn (bf16).
int launch_grouped_ffn_bf16_pair(const dsca_ffn_args* f, int num_sms, cudaStream_t stream);
// 2-D byte tensor map (e4m3 weights or two-term token rows), box = box_rows x 128, 128B swizzle.
int make_map_e4m3(CUtensorMap* m, const void* base, uint64_t rows, uint64_t cols, uint32_t box_rows);
// GEMM1 of the f8_split FFN on single-CTA tiles (gemm_sm100.cu).
int launch_gemm1_f8_single(const dsca_ffn_args* f, int num_sms, cudaStream_t stream);
// dsca_grouped_ffn with fp8-e4m3 weights and two-term e4m3 tokens (f8_split = 1).
int launch_grouped_ffn_f8_split(const dsca_ffn_args* f, int num_sms, cudaStream_t stream);
// One warp per row: bf16 rows -> two-term e4m3 rows and 1 / s (fp8_split.cuh).
int launch_split_rows(const void* src, int ld, int rows, const int32_t* rows_dev, int K, void* dst, float* inv_scale,
                      cudaStream_t stream);

}  // namespace dsca
