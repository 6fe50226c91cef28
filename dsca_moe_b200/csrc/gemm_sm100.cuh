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

enum Epi { kEpiSwiGLU = 0, kEpiReLU = 1, kEpiStore = 2 };

// One GEMM segment: the routed experts (row groups with device-side offsets) or the shared
// expert (one group over all tokens).  "b" is the weight operand: [groups * b_rows_per_group, K].
struct Segment {
  const int32_t* group_offsets;  // device [ngroups + 1], or null = one group of `rows`
  const int32_t* group_weight;   // device [ngroups], or null = identity
  int ngroups;
  int rows;
  int n_tiles;                   // 256-wide blocks of weight rows per group
  int b_rows_per_group;
  int k_blocks;
  __nv_bfloat16* c;
  int ldc;
  int n_store;
  int capacity;
  // expert parallel: when set, output row r of group e belongs to chunk (src, e) of the
  // receive buffer and is stored straight into rank src's return buffer (peer memory)
  const ep::Ctx* ep;
};

struct Params {
  Segment seg[2];
  int nseg;
  int seg_first;  // segment whose tiles come first
  int epi;
  int32_t* err;
  ep::Ctx* ep_signal;  // set: signal the return flag at every peer once the grid is done
};

// A tile: token rows [row0, row0 + rows_valid) of group `group`, weight rows [b_row0, b_row0 + 256)
// (weight block n_blk of the group).
struct TileInfo {
  int seg, group, row0, rows_valid, b_row0, n_blk;
};

// Destination row pointer of a routed output row in the expert-parallel return path.
__device__ __forceinline__ __nv_bfloat16* ep_return_row(const ep::Ctx* c, int e, int r, int ldc) {
  for (int src = 0; src < c->G; ++src) {
    const int cs = c->chunk_start[e][src];
    if (r >= cs && r < cs + c->chunk_len[e][src])
      return reinterpret_cast<__nv_bfloat16*>(c->ret[src]) + (size_t)(c->ret_start[e][src] + r - cs) * ldc;
  }
  return nullptr;
}

struct SmemCtl {
  uint64_t full[kMaxStages];
  uint64_t empty[kMaxStages];
  uint64_t tmem_full[2];
  uint64_t tmem_empty[2];
  uint64_t mma_done;
  uint32_t tmem_base;
  int abort_flag;
  int total_tiles;
  int cls_start[5];              // tile classes in schedule order (see build_group_table)
  int cls_kind[4];               // 0 / 1: full tiles of segment 0 / 1; 2 / 3: tail tiles
  int full_start[kMaxGroups + 1];  // segment 0: prefix of full-height tiles per group
  int tail_start[kMaxGroups + 1];  // segment 0: prefix of the partial tile per group
  int goff[kMaxGroups + 1];
  int gw[kMaxGroups];
};

// Tile schedule.  Tiles fall in four classes: full-height tiles (TBM token rows) of each
// segment and the partial last tile of each group.  They are laid out cost first: full tiles of
// the segment with the longer K (p.seg_first), full tiles of the other, then the partial tiles in
// the same segment order; unit u of U takes tiles in boustrophedon order (round r: r U + u for
// even r, r U + U - 1 - u for odd r), which evens out the per-unit work.  Built by one warp from
// the device-side group offsets (no host sync).
template <int TBM>
__device__ __forceinline__ void build_group_table(const Params& p, SmemCtl& ctl, int lane) {
  const Segment& sg = p.seg[0];
  const int ng = sg.ngroups;
  for (int g = lane; g <= ng; g += 32)
    ctl.goff[g] = sg.group_offsets ? sg.group_offsets[g] : (g == 0 ? 0 : sg.rows);
  for (int g = lane; g < ng; g += 32) ctl.gw[g] = sg.group_weight ? sg.group_weight[g] : g;
  __syncwarp();
  // each lane scans a contiguous run of groups, then warp scans stitch the runs
  const int per = (ng + 31) / 32;
  const int g0 = min(ng, lane * per), g1 = min(ng, g0 + per);
  auto rows_of = [&](int g) {
    int r = ctl.goff[g + 1] - ctl.goff[g];
    if (r < 0 || ctl.goff[g + 1] > sg.capacity) r = -1;
    return r;
  };
  int run_f = 0, run_t = 0;
  for (int g = g0; g < g1; ++g) {
    int r = rows_of(g);
    if (r < 0) {
      record_error(p.err, kErrCapacity);
      r = 0;
    }
    run_f += (r / TBM) * sg.n_tiles;
    run_t += (r % TBM ? 1 : 0) * sg.n_tiles;
  }
  int inc_f = run_f, inc_t = run_t;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const int vf = __shfl_up_sync(0xffffffffu, inc_f, off), vt = __shfl_up_sync(0xffffffffu, inc_t, off);
    if (lane >= off) {
      inc_f += vf;
      inc_t += vt;
    }
  }
  int ex_f = inc_f - run_f, ex_t = inc_t - run_t;
  for (int g = g0; g < g1; ++g) {
    ctl.full_start[g] = ex_f;
    ctl.tail_start[g] = ex_t;
    const int r = max(0, rows_of(g));
    ex_f += (r / TBM) * sg.n_tiles;
    ex_t += (r % TBM ? 1 : 0) * sg.n_tiles;
  }
  const int tot_f = __shfl_sync(0xffffffffu, inc_f, 31), tot_t = __shfl_sync(0xffffffffu, inc_t, 31);
  if (lane == 0) {
    ctl.full_start[ng] = tot_f;
    ctl.tail_start[ng] = tot_t;
    int cnt[4] = {tot_f, 0, tot_t, 0};  // by kind
    if (p.nseg > 1) {
      const Segment& s1 = p.seg[1];
      cnt[1] = (s1.rows / TBM) * s1.n_tiles;
      cnt[3] = (s1.rows % TBM ? 1 : 0) * s1.n_tiles;
    }
    const int L = p.seg_first;
    const int kinds[4] = {L, 1 - L, 2 + L, 3 - L};
    int acc = 0;
    for (int c = 0; c < 4; ++c) {
      ctl.cls_kind[c] = kinds[c];
      ctl.cls_start[c] = acc;
      acc += cnt[kinds[c]];
    }
    ctl.cls_start[4] = acc;
    ctl.total_tiles = acc;
  }
}

// Tile index of round r for unit u of U (boustrophedon order).
__device__ __forceinline__ int sched_tile(int r, int u, int U) { return r * U + ((r & 1) ? U - 1 - u : u); }

template <int TBM>
__device__ __forceinline__ TileInfo decode(const Params& p, const SmemCtl& s, int tile) {
  TileInfo ti;
  int c = 0;
  while (c < 3 && tile >= s.cls_start[c + 1]) ++c;
  const int kind = s.cls_kind[c];
  const int local = tile - s.cls_start[c];
  const bool tail = kind >= 2;
  const int seg = kind & 1;
  const Segment& sg = p.seg[seg];
  ti.seg = seg;
  if (seg == 0) {
    const int* start = tail ? s.tail_start : s.full_start;
    int lo = 0, hi = sg.ngroups;  // g with start[g] <= local < start[g + 1]
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (start[mid] <= local) lo = mid; else hi = mid;
    }
    const int g = lo;
    const int l = local - start[g];
    const int rows_g = s.goff[g + 1] - s.goff[g];
    const int m_blk = tail ? rows_g / TBM : l / sg.n_tiles;
    ti.n_blk = tail ? l : l - m_blk * sg.n_tiles;
    ti.group = g;
    ti.row0 = s.goff[g] + m_blk * TBM;
    ti.rows_valid = tail ? rows_g - m_blk * TBM : TBM;
    ti.b_row0 = s.gw[g] * sg.b_rows_per_group + ti.n_blk * BN;
  } else {
    const int m_blk = tail ? sg.rows / TBM : local / sg.n_tiles;
    ti.n_blk = tail ? local : local - m_blk * sg.n_tiles;
    ti.group = 0;
    ti.row0 = m_blk * TBM;
    ti.rows_valid = tail ? sg.rows - m_blk * TBM : TBM;
    ti.b_row0 = ti.n_blk * BN;
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

}  // namespace dsca
