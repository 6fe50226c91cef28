// K5 — grouped expert GEMM on CTA pairs (tcgen05 cta_group::2), weights as the M operand.
//
// Same contract as gemm_sm100.cu (routed experts with device-side row offsets + the shared
// expert, SwiGLU / ReLU / store epilogues, expert-parallel remote store), computed as
// C^T = W . X^T: a tile is 256 weight rows (M) x up to 256 token rows (N) x K.
//   * A cluster of two CTAs on neighbouring SMs runs tcgen05.mma.cta_group::2 (M256 N<=256 K16)
//     issued by the even CTA.  Each CTA loads its own 128 weight rows and its half of the token
//     rows, so an SM streams at most 32 KB per 64-wide K step (48 KB for a 128 x 256 single-CTA
//     tile of the same tensor work).
//   * The token count of a tile is rounded up to 16 only (the MMA N granularity), not to a tile
//     height: an expert with 300 routed rows costs 256 + 48 token columns instead of 2 x 256
//     rows.
//   * Accumulator (per CTA): TMEM lane = weight row, column = token.  The epilogue writes each
//     token's outputs as 64-byte row pieces (32 consecutive channels), staged per warp in
//     shared memory and written as 16-byte pieces.  SwiGLU: weights are packed in 256-row
//     blocks [128 gate | 128 up]; a CTA loads the gate and the up rows of its 128 channels and
//     runs two MMAs per K step into a gate and an up accumulator (N <= 128), so SiLU(g) * u is
//     formed in registers.
//   warp 0      TMA producer (one thread), 128-byte swizzle, 6-stage ring.  No multicast.
//   warp 1      TMEM allocator (512 columns, two accumulators); in the even CTA the MMA issuer.
//   warps 2-5   epilogue.
// Both CTAs' loads complete on the even CTA's full barrier; the even CTA's commits arrive on the
// empty / accumulator-full barriers of both CTAs; each epilogue warp arrives on the even CTA's
// accumulator-empty barrier.  Every wait is bounded (2 s); on a timeout the kernel records
// DSCA_ERR_WAIT_TIMEOUT, drains what it can observe, waits a bounded grace period for copies
// completing on the peer's barriers, frees TMEM and returns.
#include <algorithm>

#include "gemm_sm100.cuh"

#ifndef DSCA_GEMM2_WIDE_STAGES
#define DSCA_GEMM2_WIDE_STAGES 1
#endif

namespace dsca {
namespace gemm {
namespace pair {

// Per-epilogue configuration.  SwiGLU: a CTA's 128 channels need 128 gate rows (slot A) and the
// 128 matching up rows (slot A2), two MMAs per K step into a gate and an up accumulator of N <=
// 128 columns each.  Others: 128 weight rows (slot A), N <= 256.
//
// F8 (fp8-e4m3 weights): a stage is 128 bytes of K per row as in bf16 — 128 e4m3 weights instead
// of 64 bf16 — and the tokens come as two e4m3 planes (hi, lo; fp8_split.cuh), so each 32-byte K
// step runs two tcgen05.mma.kind::f8f6f4 (W . hi, W . lo) into the same accumulator: the tensor
// time per K element of the bf16 MMA, half its weight bytes, and no conversion of the weights.
// The epilogue multiplies by the weight row's scale and the token row's 1 / s.
// F8 SwiGLU takes up to 256 tokens a tile (an expert's rows in one tile up to 256, so each weight
// block is streamed once): its gate and up accumulators fill the 512 TMEM columns, one buffer.
//
// kEpiSwiGLU2 (bf16): a tile is the 128 channels of one packed 256-row block [128 gate | 128 up]
// times up to 256 tokens.  CTA r loads gate rows 64 r + [0, 64) and the matching up rows as one
// 128-row operand (two 64-row boxes), so one M256 MMA per K16 step fills a single accumulator
// whose TMEM lanes 0-63 are gate and 64-127 up values of the same 64 channels: an SM streams 32
// KB per K step (16 KB weights + 16 KB tokens) for the tensor work a 128 x 256 single-CTA tile
// does with 48 KB.  The epilogue warps of lane quarters q and q + 2 hold the gate and the up
// values of 32 channels; per chunk of 32 tokens each sends the other the values of the 16
// tokens the other forms SiLU(g) * u for (16 x 32 fp32 each way, two buffers per warp pair,
// mbarrier-paced), so both warps compute and store at once.
//
// kWide (bf16 store epilogue, GEMM2): a stage holds two 64-wide K blocks of each operand (two
// TMA boxes each, 64 KB per CTA, 3 stages), eight MMAs per full-barrier wait and commit.
template <int EPI, bool F8 = false>
struct Cfg {
  static constexpr bool kGlu = EPI == kEpiSwiGLU;
  static constexpr bool kG2 = EPI == kEpiSwiGLU2;
  static constexpr bool kWide = (EPI == kEpiStore || EPI == kEpiSwiGLU2) && !F8 && DSCA_GEMM2_WIDE_STAGES;
  static constexpr int kSub = kWide ? 2 : 1;              // 128-byte K boxes per operand and stage
  static constexpr int TBN = (kGlu && !F8) ? 128 : 256;  // token rows per tile (MMA N)
  static constexpr int kAccBufs = (kGlu && F8) ? 1 : 2;  // accumulator buffers (256 columns each)
  static constexpr int kUpCol = kGlu ? TBN : 0;          // SwiGLU: the up accumulator's column
  static constexpr int S = F8 ? (kGlu ? 3 : 4) : (kGlu ? 5 : (kWide ? 3 : 6));  // stages
  static_assert(!kWide || S * (128 * 128 * 2 * 2) + 4 * 32 * 32 * 2 + (kG2 ? 16384 : 0) + 1024 <= 227 * 1024,
                "two-box stages exceed the shared memory of a CTA");
  static constexpr int kWBox = kG2 ? 64 : 128;            // weight rows per TMA box
  static constexpr int kTBox = TBN / 2;                   // token rows per TMA box
  static constexpr int kKE = F8 ? 128 : BK;               // K elements per box (128 bytes a row)
  static constexpr int kKS = kKE * kSub;                  // K elements per stage
  static constexpr int kABytes = 128 * 128 * kSub;        // 16 KB per box
  static constexpr int kA2Bytes = kGlu ? 128 * 128 : 0;
  static constexpr int kTPlane = (TBN / 2) * 128 * kSub;  // this CTA's token rows, one plane
  static constexpr int kTBytes = (F8 ? 2 : 1) * kTPlane;
  static constexpr int kStageBytes = kABytes + kA2Bytes + kTBytes;
  static constexpr int kStageElems = 32 * 32;             // epilogue staging per warp, bf16
  static constexpr int kXBytes = kG2 ? 2 * 2 * 32 * 32 * 4 : 0;  // gate / up exchange, fp32
  static constexpr int kSmemBytes = S * kStageBytes + 4 * kStageElems * 2 + kXBytes + 1024;
};

// MMA N for a tile of `ntok` token rows: a multiple of 16 (each CTA holds N / 2 rows, a whole
// number of 8-row swizzle atoms).
__device__ __forceinline__ int tile_n(int ntok) { return max(16, (ntok + 15) & ~15); }

// D(tmem) (+)= A(smem desc) * B(smem desc), e4m3 x e4m3, fp32 accumulate, CTA pair
__device__ __forceinline__ void umma_f8_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                             uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

template <int EPI, bool F8>
__global__ void __launch_bounds__(kThreads, 1)
    pair_gemm_kernel(const __grid_constant__ CUtensorMap tmW0, const __grid_constant__ CUtensorMap tmT0,
                     const __grid_constant__ CUtensorMap tmW1, const __grid_constant__ CUtensorMap tmT1,
                     const Params p) {
  using C = Cfg<EPI, F8>;
  constexpr int S = C::S;
  constexpr int TBN = C::TBN;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  __shared__ SmemCtl ctl;
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t smem_a = smem_u32(smem);
  const uint32_t smem_a2 = smem_a + S * C::kABytes;
  const uint32_t smem_t = smem_a2 + S * C::kA2Bytes;
  __nv_bfloat16* stage_all = reinterpret_cast<__nv_bfloat16*>(smem + S * C::kStageBytes);
  float* xbuf = reinterpret_cast<float*>(smem + S * C::kStageBytes + 4 * C::kStageElems * 2);

  const int warp = warp_id(), lane = lane_id();
  volatile int* abort_flag = &ctl.abort_flag;
  const uint32_t rank = cluster_ctarank();  // 0 = the CTA that issues the MMAs
  pdl_launch_dependents();  // a programmatic dependent (the combine) may be scheduled early
  const int unit = (int)(blockIdx.x >> 1), units = (int)(gridDim.x >> 1);

  // ---- prologue: barriers, TMEM, tile schedule
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(smem_u32(&ctl.full[s]), 1);
      mbar_init(smem_u32(&ctl.empty[s]), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(smem_u32(&ctl.tmem_full[a]), 1);
      mbar_init(smem_u32(&ctl.tmem_empty[a]), 8);  // 4 epilogue warps x 2 CTAs
    }
    // the tile queue: the even CTA's producer publishes each tile id into both CTAs' queues;
    // its readers (the even CTA's MMA thread and epilogue warps, the odd CTA's producer and
    // epilogue warps) release a slot on the even CTA's tq_empty
    for (int i = 0; i < kTQ; ++i) {
      mbar_init(smem_u32(&ctl.tq_full[i]), 1);
      mbar_init(smem_u32(&ctl.tq_empty[i]), 10);
    }
    mbar_init(smem_u32(&ctl.mma_done), 1);
    for (int i = 0; i < 2; ++i)
      for (int b = 0; b < 2; ++b)
        for (int d = 0; d < 2; ++d) {
          mbar_init(smem_u32(&ctl.xfull[i][b][d]), 1);
          mbar_init(smem_u32(&ctl.xempty[i][b][d]), 1);
        }
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
    tmem_alloc_pair(smem_u32(&ctl.tmem_base), kTmemCols);
    tmem_relinquish_pair();
  }
  if (warp == 2) build_group_table<TBN>(p, ctl, lane);
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // both CTAs' barriers exist before any cross-CTA signal
  tc_fence_after();
  const uint32_t tmem_base = ctl.tmem_base;
  const int total = ctl.total_tiles;

  if (warp == 0) {
    // ---------------- TMA producer: this CTA's weight rows and its half of the token rows
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0;
      int pending_phase[S];
      for (int i = 0; i < S; ++i) pending_phase[i] = -1;
      bool ok = true;
      // GEMM2 after GEMM1: griddepcontrol.wait (GEMM1 has completed) before the first load, or,
      // with the shared-expert handoff, before the first routed tile's load and the handoff
      // flag before the first shared-expert tile's
      bool all_ready = !p.pdl_wait_all;
      if (!all_ready && p.seg1_flag == nullptr) {
        pdl_wait();
        all_ready = true;
      }
      bool seg1_ready = all_ready;
      bool seg0_ready = !p.pdl_seg0_wait;
      const uint64_t pol_first = l2_policy_evict_first(), pol_last = l2_policy_evict_last();
      uint32_t tq_empty0[kTQ];
      for (int i = 0; i < kTQ; ++i) tq_empty0[i] = mapa_shared(smem_u32(&ctl.tq_empty[i]), 0);
      // the tile of round r: the even CTA draws it and publishes it to both CTAs' queues (the id
      // into the odd CTA's queue by an asynchronous store that completes on its barrier); -1
      // past the last tile, -2 when the wait for a free queue slot gave up
      auto publish = [&](int r) -> int {
        const int slot = r % kTQ;
        if (!mbar_wait<true>(smem_u32(&ctl.tq_empty[slot]), (uint32_t)(((r / kTQ) & 1) ^ 1), abort_flag, p.err))
          return -2;
        int tile = ticket_tile(p, r, unit, units);
        if (tile >= total) tile = -1;
        *reinterpret_cast<volatile int*>(&ctl.tq[slot]) = tile;
        mbar_arrive(smem_u32(&ctl.tq_full[slot]));
        const uint32_t rbar = mapa_shared(smem_u32(&ctl.tq_full[slot]), 1);
        mbar_arrive_expect_tx_remote(rbar, 4u);
        st_async_s32(mapa_shared(smem_u32(&ctl.tq[slot]), 1), tile, rbar);
        return tile;
      };
      int next = rank == 0 ? publish(0) : 0;
      for (int r = 0; ok; ++r) {
        int tile;
        if (rank == 0) {
          if (next == -2) {
            ok = false;
            break;
          }
          tile = next;
          // the next round's tile is drawn one tile ahead (its ticket latency overlaps this
          // tile's loads)
          if (tile >= 0) next = publish(r + 1);
        } else {
          tile = tq_take<true>(ctl, r, abort_flag, p.err, tq_empty0);
          if (tile < 0 && *abort_flag) ok = false;
        }
        if (tile < 0) break;
        const TileInfo ti = decode<TBN>(p, ctl, tile);
        if (ti.seg == 0 && !seg0_ready) {
          pdl_wait();  // the preceding kernel (the permute) has written the routed rows
          seg0_ready = true;
        }
        if (!all_ready && ti.seg == 0) {
          pdl_wait();  // GEMM1 has completed
          all_ready = seg1_ready = true;
        }
        if (!seg1_ready && ti.seg == 1) {
          if (!wait_seg1_flag(p, abort_flag)) {
            ok = false;
            break;
          }
          seg1_ready = true;
        }
        const CUtensorMap* mw = ti.seg == 0 ? &tmW0 : &tmW1;
        const CUtensorMap* mt = ti.seg == 0 ? &tmT0 : &tmT1;
        const int half = tile_n(ti.rows_valid) / 2;
        // the whole token box lands every stage (rows past the tile's tokens are loaded and not
        // used by the MMA)
        constexpr uint32_t tx = 2u * (uint32_t)C::kStageBytes;
        // weight rows: SwiGLU packs 256-row blocks [128 gate | 128 up]; this CTA's 128 channels
        // are packed block 2 n_blk + rank
        // kEpiSwiGLU2: gate rows 64 rank + [0, 64) of the tile's 256-row block (the up rows 128 further)
        const int w_row = C::kGlu ? ti.b_row0 + ti.n_blk * BN + 256 * (int)rank
                                  : ti.b_row0 + (C::kG2 ? 64 : 128) * (int)rank;
        const int t_row = ti.row0 + half * (int)rank;
        const int kb_n = p.seg[ti.seg].k_blocks;
        // hybrid full tile (SwiGLU): this CTA's 128 tokens (two 64-row token boxes into slot A)
        // and the gate (even CTA) or up (odd CTA) rows of the tile's 128 channels (slot A2)
        const bool full = !F8 && C::kGlu && ti.full;
        const int f_trow = ti.row0 + 128 * (int)rank, f_wrow = ti.b_row0 + 128 * (int)rank;
        constexpr uint32_t tx_full = 2u * (uint32_t)(C::kABytes + C::kA2Bytes);
        // routed swap-AB tile: L2 prefetch of this CTA's boxes beyond the shared-memory stages,
        // then one K block l2_ahead ahead of every load
        const int pf = (ti.seg == 0 && !full) ? p.l2_ahead : 0;
        auto prefetch_kb = [&](int k) {
          for (int h = 0; h < C::kSub; ++h) {
            const int kx = k * C::kKS + h * C::kKE;
            tma_prefetch_l2_2d(mw, kx, w_row);
            if constexpr (C::kGlu || C::kG2) tma_prefetch_l2_2d(mw, kx, w_row + 128);
            tma_prefetch_l2_2d(mt, kx, t_row);
          }
        };
        for (int kb = S; kb < min(pf, kb_n); ++kb) prefetch_kb(kb);
        for (int kb = 0; kb < kb_n; ++kb) {
          if (!mbar_wait(smem_u32(&ctl.empty[s]), ph ^ 1u, abort_flag, p.err)) { ok = false; break; }
          const uint32_t fb = smem_u32(&ctl.full[s]);
          const uint32_t fb0 = mapa_shared(fb, 0);  // the even CTA's full barrier
          if (pf > 0 && kb + pf < kb_n && kb + pf >= S) prefetch_kb(kb + pf);
          // L2 policies (Params::l2_hints): routed weights evict-first, the rest evict-last
          const uint64_t wpol = ti.seg == 0 ? pol_first : pol_last;
          if (full) {
            if (rank == 0) mbar_arrive_expect_tx(fb, tx_full);
            if (p.l2_hints) {
              tma_load_2d_pair_hint(smem_a + s * C::kABytes, mt, fb0, kb * C::kKE, f_trow, pol_last);
              tma_load_2d_pair_hint(smem_a + s * C::kABytes + C::kABytes / 2, mt, fb0, kb * C::kKE, f_trow + 64, pol_last);
              tma_load_2d_pair_hint(smem_a2 + s * C::kA2Bytes, mw, fb0, kb * C::kKE, f_wrow, wpol);
            } else {
              tma_load_2d_pair(smem_a + s * C::kABytes, mt, fb0, kb * C::kKE, f_trow);
              tma_load_2d_pair(smem_a + s * C::kABytes + C::kABytes / 2, mt, fb0, kb * C::kKE, f_trow + 64);
              tma_load_2d_pair(smem_a2 + s * C::kA2Bytes, mw, fb0, kb * C::kKE, f_wrow);
            }
          } else if constexpr (C::kWide) {
            if (rank == 0) mbar_arrive_expect_tx(fb, tx);
            // two 64-wide K boxes of weights and tokens; a box past K reads zeros
#pragma unroll
            for (int h = 0; h < C::kSub; ++h) {
              const int kx = kb * C::kKS + h * C::kKE;
              const uint32_t wdst = smem_a + s * C::kABytes + h * (C::kABytes / C::kSub);
              const uint32_t tdst = smem_t + s * C::kTBytes + h * (C::kTPlane / C::kSub);
              // kEpiSwiGLU2: the gate rows, then the up rows 128 further, as the box's rows 64-127
              constexpr uint32_t up_off = C::kABytes / C::kSub / 2;
              if (p.l2_hints) {
                tma_load_2d_pair_hint(wdst, mw, fb0, kx, w_row, wpol);
                if constexpr (C::kG2) tma_load_2d_pair_hint(wdst + up_off, mw, fb0, kx, w_row + 128, wpol);
                tma_load_2d_pair_hint(tdst, mt, fb0, kx, t_row, pol_last);
              } else {
                tma_load_2d_pair(wdst, mw, fb0, kx, w_row);
                if constexpr (C::kG2) tma_load_2d_pair(wdst + up_off, mw, fb0, kx, w_row + 128);
                tma_load_2d_pair(tdst, mt, fb0, kx, t_row);
              }
            }
          } else {
            if (rank == 0) mbar_arrive_expect_tx(fb, tx);
            if (p.l2_hints) {
              tma_load_2d_pair_hint(smem_a + s * C::kABytes, mw, fb0, kb * C::kKE, w_row, wpol);
              if constexpr (C::kGlu)
                tma_load_2d_pair_hint(smem_a2 + s * C::kA2Bytes, mw, fb0, kb * C::kKE, w_row + 128, wpol);
              if constexpr (C::kG2)  // the up rows as the operand's rows 64-127
                tma_load_2d_pair_hint(smem_a + s * C::kABytes + C::kABytes / 2, mw, fb0, kb * C::kKE, w_row + 128,
                                      wpol);
              tma_load_2d_pair_hint(smem_t + s * C::kTBytes, mt, fb0, kb * C::kKE, t_row, pol_last);
              if constexpr (F8)  // the lo plane of the same token rows
                tma_load_2d_pair_hint(smem_t + s * C::kTBytes + C::kTPlane, mt, fb0,
                                      p.seg[ti.seg].t_lo + kb * C::kKE, t_row, pol_last);
            } else {
              tma_load_2d_pair(smem_a + s * C::kABytes, mw, fb0, kb * C::kKE, w_row);
              if constexpr (C::kGlu) tma_load_2d_pair(smem_a2 + s * C::kA2Bytes, mw, fb0, kb * C::kKE, w_row + 128);
              if constexpr (C::kG2)
                tma_load_2d_pair(smem_a + s * C::kABytes + C::kABytes / 2, mw, fb0, kb * C::kKE, w_row + 128);
              tma_load_2d_pair(smem_t + s * C::kTBytes, mt, fb0, kb * C::kKE, t_row);
              if constexpr (F8)
                tma_load_2d_pair(smem_t + s * C::kTBytes + C::kTPlane, mt, fb0, p.seg[ti.seg].t_lo + kb * C::kKE,
                                 t_row);
            }
          }
          pending_phase[s] = (int)ph;
          if (++s == S) { s = 0; ph ^= 1u; }
        }
      }
      // every CTA completes only after GEMM1 (a CTA that ran only shared-expert tiles under the
      // handoff has not waited for it yet), so later work ordered after GEMM2 is after GEMM1 too
      if (!all_ready) pdl_wait();
      if (!ok && rank == 0) {
        // drain: the last armed phase of every stage must complete before the CTA exits (this
        // also covers the odd CTA's loads, which complete on these barriers)
        for (int i = 0; i < S; ++i)
          if (pending_phase[i] >= 0) mbar_drain(smem_u32(&ctl.full[i]), (uint32_t)pending_phase[i]);
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer (even CTA)
    if (lane == 0 && rank == 0) {
      constexpr uint32_t idesc_m = F8 ? idesc_e4m3_f32(256, 0) : idesc_bf16_f32(256, 0);
      int s = 0;
      uint32_t ph = 0;
      int it = 0;
      bool ok = true;
      for (int r = 0; ok; ++r, ++it) {
        const int tile = tq_take<false>(ctl, r, abort_flag, p.err, nullptr);
        if (tile < 0) {
          ok = *abort_flag == 0;
          break;
        }
        const TileInfo ti = decode<TBN>(p, ctl, tile);
        const bool full = !F8 && C::kGlu && ti.full;
        const uint32_t idesc = full ? idesc_bf16_f32(256, 256)
                                    : (idesc_m | ((uint32_t)(tile_n(ti.rows_valid) >> 3) << 17));
        const int acc = it % C::kAccBufs;
        const uint32_t acc_ph = (uint32_t)((it / C::kAccBufs) & 1);
        if (!mbar_wait(smem_u32(&ctl.tmem_empty[acc]), acc_ph ^ 1u, abort_flag, p.err)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(acc * 256);
        const int kb_n = p.seg[ti.seg].k_blocks;
        for (int kb = 0; kb < kb_n; ++kb) {
          if (!mbar_wait(smem_u32(&ctl.full[s]), ph, abort_flag, p.err)) { ok = false; break; }
          tc_fence_after();
          const uint64_t adesc = sw128_kmajor_desc(smem_a + s * C::kABytes);
          const uint64_t tdesc = sw128_kmajor_desc(smem_t + s * C::kTBytes);
          if (full) {
            // tokens (slot A, M = 256 over the pair) x [gate | up] rows of 128 channels (slot
            // A2, N = 256 over the pair): TMEM lane = token, columns 0-127 gate, 128-255 up
            const uint64_t wdesc = sw128_kmajor_desc(smem_a2 + s * C::kA2Bytes);
#pragma unroll
            for (int k = 0; k < BK / 16; ++k)
              umma_f16_pair(d_tmem, adesc + (uint64_t)(2 * k), wdesc + (uint64_t)(2 * k), idesc,
                            (kb > 0 || k > 0) ? 1u : 0u);
          } else if constexpr (F8) {
            // two e4m3 MMAs per 32-byte K step: the weights times the hi and the lo token plane
            const uint64_t ldesc = sw128_kmajor_desc(smem_t + s * C::kTBytes + C::kTPlane);
#pragma unroll
            for (int k = 0; k < C::kKE / 32; ++k) {
              const uint32_t accum = (kb > 0 || k > 0) ? 1u : 0u;
              const uint64_t ko = (uint64_t)(2 * k);
              umma_f8_pair(d_tmem, adesc + ko, tdesc + ko, idesc, accum);
              umma_f8_pair(d_tmem, adesc + ko, ldesc + ko, idesc, 1u);
              if constexpr (C::kGlu) {
                const uint64_t udesc = sw128_kmajor_desc(smem_a2 + s * C::kA2Bytes);
                umma_f8_pair(d_tmem + C::kUpCol, udesc + ko, tdesc + ko, idesc, accum);
                umma_f8_pair(d_tmem + C::kUpCol, udesc + ko, ldesc + ko, idesc, 1u);
              }
            }
          } else if constexpr (C::kWide) {
#pragma unroll
            for (int h = 0; h < C::kSub; ++h) {
              const uint64_t ah = sw128_kmajor_desc(smem_a + s * C::kABytes + h * (C::kABytes / C::kSub));
              const uint64_t th = sw128_kmajor_desc(smem_t + s * C::kTBytes + h * (C::kTPlane / C::kSub));
#pragma unroll
              for (int k = 0; k < BK / 16; ++k)
                umma_f16_pair(d_tmem, ah + (uint64_t)(2 * k), th + (uint64_t)(2 * k), idesc,
                              (kb > 0 || h > 0 || k > 0) ? 1u : 0u);
            }
          } else {
#pragma unroll
            for (int k = 0; k < BK / 16; ++k) {
              const uint32_t accum = (kb > 0 || k > 0) ? 1u : 0u;
              umma_f16_pair(d_tmem, adesc + (uint64_t)(2 * k), tdesc + (uint64_t)(2 * k), idesc, accum);
              if constexpr (C::kGlu) {
                const uint64_t udesc = sw128_kmajor_desc(smem_a2 + s * C::kA2Bytes);
                umma_f16_pair(d_tmem + 128, udesc + (uint64_t)(2 * k), tdesc + (uint64_t)(2 * k), idesc, accum);
              }
            }
          }
          const uint32_t eb = smem_u32(&ctl.empty[s]);
          umma_commit_pair_both(eb);
          if (++s == S) { s = 0; ph ^= 1u; }
        }
        if (!ok) break;
        const uint32_t fb = smem_u32(&ctl.tmem_full[acc]);
        umma_commit_pair_both(fb);
      }
      if (!ok) {
        // aborting: wait until every MMA this thread issued has completed before TMEM is freed
        umma_commit_pair(mapa_shared(smem_u32(&ctl.mma_done), 0));
        mbar_drain(smem_u32(&ctl.mma_done), 0);
      }
    }
  } else {
    // ---------------- epilogue (warps 2..5 -> TMEM lane quarters 2, 3, 0, 1)
    const int q = warp & 3;
    const uint32_t empty_bar[2] = {mapa_shared(smem_u32(&ctl.tmem_empty[0]), 0),
                                   mapa_shared(smem_u32(&ctl.tmem_empty[1]), 0)};
    __nv_bfloat16* stg = stage_all + (warp - 2) * C::kStageElems;
    uint32_t tq_empty0[kTQ];
    for (int i = 0; i < kTQ; ++i) tq_empty0[i] = mapa_shared(smem_u32(&ctl.tq_empty[i]), 0);
    int it = 0;
    uint32_t xg = 0;  // kEpiSwiGLU2: exchange chunks so far (the same sequence in both warps of a pair)
    for (int r = 0;; ++r, ++it) {
      int tile = 0;
      if (lane == 0)
        tile = rank == 0 ? tq_take<false>(ctl, r, abort_flag, p.err, nullptr)
                         : tq_take<true>(ctl, r, abort_flag, p.err, tq_empty0);
      tile = __shfl_sync(0xffffffffu, tile, 0);
      if (tile < 0) break;
      const TileInfo ti = decode<TBN>(p, ctl, tile);
      const Segment& sg = p.seg[ti.seg];
      const int acc = it % C::kAccBufs;
      const uint32_t acc_ph = (uint32_t)((it / C::kAccBufs) & 1);
      // one lane polls, the warp follows its verdict (tcgen05.ld below must not diverge)
      int w_ok = 1;
      if (lane == 0) w_ok = mbar_wait(smem_u32(&ctl.tmem_full[acc]), acc_ph, abort_flag, p.err) ? 1 : 0;
      w_ok = __shfl_sync(0xffffffffu, w_ok, 0);
      if (!w_ok) break;
      tc_fence_after();
      const uint32_t taddr = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * 256);
      if constexpr (C::kG2) {
        // lane quarters 0 / 1: gate values of channels 32 pr + lane (pr = q & 1) of this CTA's 64;
        // quarters 2 / 3: their up values.  Chunk of 32 tokens: the gate warp forms SiLU(g) * u
        // for tokens 0-15 and the up warp for tokens 16-31, each sending the other the 16 values
        // it lacks, then stores its 16 tokens' 64-byte row pieces.
        const int ntok = ti.rows_valid;
        const int ncol = tile_n(ntok);
        const int pr = q & 1;
        const int me = q >> 1, other = me ^ 1;  // 0 = gate warp, 1 = up warp
        const int keep = me * 16;  // this warp's tokens: chunk columns keep + [0, 16)
        const int ch0 = ti.n_blk * 128 + 64 * (int)rank + 32 * pr;
        bool x_ok = true;
#pragma unroll 1
        for (int c = 0; c < ncol; c += 32, ++xg) {
          const uint32_t b = xg & 1u, use = xg >> 1;
          float* xs = xbuf + ((pr * 2 + (int)b) * 2 + me) * 512;     // this warp's sent half
          float* xr = xbuf + ((pr * 2 + (int)b) * 2 + other) * 512;  // the other warp's
          uint32_t v[32];
          tmem_ld32(taddr + c, v);
          tmem_wait_ld();
          // every lane waits: the other warp has read this buffer's previous use of our half
          bool w = use == 0 || mbar_wait(smem_u32(&ctl.xempty[pr][b][me]), (use - 1u) & 1u, abort_flag, p.err);
          if (!__all_sync(0xffffffffu, w)) { x_ok = false; break; }
#pragma unroll
          for (int j = 0; j < 16; ++j) xs[j * 32 + lane] = __uint_as_float(me ? v[j] : v[16 + j]);
          __syncwarp();
          if (lane == 0) mbar_arrive(smem_u32(&ctl.xfull[pr][b][me]));
          w = mbar_wait(smem_u32(&ctl.xfull[pr][b][other]), use & 1u, abort_flag, p.err);
          if (!__all_sync(0xffffffffu, w)) { x_ok = false; break; }
          float o[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) o[j] = xr[j * 32 + lane];
          __syncwarp();
          if (lane == 0) mbar_arrive(smem_u32(&ctl.xempty[pr][b][other]));
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const float mine = __uint_as_float(me ? v[16 + j] : v[j]);
            const float g = me ? o[j] : mine, up = me ? mine : o[j];
            stg[j * 32 + lane] = __float2bfloat16_rn(silu(g) * up);
          }
          __syncwarp();
#pragma unroll
          for (int rr = 0; rr < 2; ++rr) {
            const int jj = rr * 8 + (lane >> 2), piece = lane & 3;
            const int t = c + keep + jj, col = ch0 + piece * 8;
            if (t < ntok && col < sg.n_store)
              *reinterpret_cast<uint4*>(sg.c + (size_t)(ti.row0 + t) * sg.ldc + col) =
                  *reinterpret_cast<const uint4*>(stg + jj * 32 + piece * 8);
          }
          __syncwarp();
        }
        if (!x_ok) break;
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_remote(empty_bar[acc]);
        // shared-expert handoff: the 8 epilogue warps of the pair count each stored tile
        if (p.seg1_done != nullptr && ti.seg == 1) seg1_tile_stored(p, ctl, lane, 8u);
        continue;
      }
      if (!F8 && C::kGlu && ti.full) {
        // hybrid full tile: TMEM lane = this CTA's token 32 q + lane, columns 0-127 gate and
        // 128-255 up of channels 128 n_blk + [0, 128): each lane stores its row's 64-byte pieces
        const size_t row = (size_t)(ti.row0 + 128 * (int)rank + q * 32 + lane);
        __nv_bfloat16* crow = sg.c + row * (size_t)sg.ldc;
        const int col0 = ti.n_blk * 128;
#pragma unroll 1
        for (int c = 0; c < 128; c += 32) {
          uint32_t g[32], u[32];
          tmem_ld32(taddr + c, g);
          tmem_ld32(taddr + 128 + c, u);
          tmem_wait_ld();
          uint32_t packed[16];
#pragma unroll
          for (int i = 0; i < 16; ++i)
            packed[i] = pack_bf16x2(silu(__uint_as_float(g[2 * i])) * __uint_as_float(u[2 * i]),
                                    silu(__uint_as_float(g[2 * i + 1])) * __uint_as_float(u[2 * i + 1]));
          const int col = col0 + c;
          if (col < sg.n_store) {
            uint4* dst = reinterpret_cast<uint4*>(crow + col);
#pragma unroll
            for (int v = 0; v < 4; ++v)
              if (col + v * 8 < sg.n_store)
                dst[v] = make_uint4(packed[4 * v], packed[4 * v + 1], packed[4 * v + 2], packed[4 * v + 3]);
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_remote(empty_bar[acc]);
        continue;
      }
      const int ntok = ti.rows_valid;
      const int ncol = tile_n(ntok);
      // this warp's 32 output channels: SwiGLU channel block n_blk (256 channels per pair);
      // otherwise weight rows of the 256-row block
      const int ch0 = ti.n_blk * 256 + 128 * (int)rank + 32 * q;
      // F8: this lane's weight row scale(s) (gate and up for SwiGLU)
      float wsc0 = 1.0f, wsc1 = 1.0f;
      if constexpr (F8) {
        const int wr = C::kGlu ? ti.b_row0 + ti.n_blk * BN + 256 * (int)rank + 32 * q + lane
                               : ti.b_row0 + 128 * (int)rank + 32 * q + lane;
        // SwiGLU: the odd CTA of a group's last tile holds no channels when ip % 256 == 128 (its
        // weight rows lie past the group's); only channels below n_store read a scale
        if (!C::kGlu || ch0 + lane < sg.n_store) {
          wsc0 = __ldg(sg.w_scale + wr);
          if constexpr (C::kGlu) wsc1 = __ldg(sg.w_scale + wr + 128);
        }
      }
      // staged output: each lane writes its channel for 32 tokens, then the warp stores whole
      // 64-byte token-row pieces with 16-byte stores
#pragma unroll 1
      for (int c = 0; c < ncol; c += 32) {
        // F8: the 1 / s of token c + lane, broadcast per token below
        float tsv = 1.0f;
        if constexpr (F8) tsv = (c + lane < ntok) ? __ldg(sg.t_scale + ti.row0 + c + lane) : 0.0f;
        uint32_t v[32];
        tmem_ld32(taddr + c, v);
        if constexpr (C::kGlu) {
          uint32_t u[32];
          tmem_ld32(taddr + C::kUpCol + c, u);
          tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            float g = __uint_as_float(v[j]), up = __uint_as_float(u[j]);
            if constexpr (F8) {
              const float ts = __shfl_sync(0xffffffffu, tsv, j);
              g = g * wsc0 * ts;
              up = up * wsc1 * ts;
            }
            stg[j * 32 + lane] = __float2bfloat16_rn(silu(g) * up);
          }
        } else {
          tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            float a = __uint_as_float(v[j]);
            if constexpr (F8) a = a * wsc0 * __shfl_sync(0xffffffffu, tsv, j);
            if constexpr (EPI == kEpiReLU) a = fmaxf(a, 0.0f);
            stg[j * 32 + lane] = __float2bfloat16_rn(a);
          }
        }
        __syncwarp();
#pragma unroll
        for (int rr = 0; rr < 4; ++rr) {
          const int jj = rr * 8 + (lane >> 2), piece = lane & 3;
          const int t = c + jj, col = ch0 + piece * 8;
          if (t < ntok && col < sg.n_store) {
            const uint4 val = *reinterpret_cast<const uint4*>(stg + jj * 32 + piece * 8);
            const int row = ti.row0 + t;
            __nv_bfloat16* crow = sg.c + (size_t)row * sg.ldc;
            if (EPI == kEpiStore && sg.ep != nullptr) {
              // expert parallel: this row goes back to the rank that sent it (NVLink store)
              crow = ep_return_row(sg.ep, ti.group, row, sg.ldc);
              if (crow == nullptr) {
                record_error(p.err, kErrIndex);
                continue;
              }
            }
            *reinterpret_cast<uint4*>(crow + col) = val;
          }
        }
        __syncwarp();
      }
      // every lane's TMEM reads are complete: the warp releases the accumulator once
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_remote(empty_bar[acc]);
    }
  }

  __syncthreads();
  if (*abort_flag) {
    // the odd CTA's loads complete on the even CTA's barriers, which this CTA cannot observe:
    // give copies still in flight a bounded grace period before the pair frees its memory
    const uint64_t t0 = globaltimer_ns();
    while (globaltimer_ns() - t0 < 200000ull) __nanosleep(1000);
  }
  cluster_sync_all();  // the pair's MMAs into this CTA's TMEM and remote arrivals are finished
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, kTmemCols);
  }
  if (threadIdx.x == 0) tile_counter_exit(p);
  if (p.ep_signal != nullptr) ep::signal_when_grid_done(p.ep_signal, &p.ep_signal->return_done, ep::kReturn);
}

}  // namespace pair
}  // namespace gemm

template <int EPI, bool F8 = false>
static int launch_pair(const CUtensorMap& w0, const CUtensorMap& t0, const CUtensorMap& w1, const CUtensorMap& t1,
                       const gemm::Params& p, int grid, cudaStream_t stream) {
  static PerDeviceOnce attr_once;
  constexpr int smem_bytes = gemm::pair::Cfg<EPI, F8>::kSmemBytes;
  auto kern = gemm::pair::pair_gemm_kernel<EPI, F8>;
  if (attr_once.run([&] {
        return cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes);
      }) != cudaSuccess)
    return DSCA_ERR_CUDA;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3(gemm::kThreads);
  cfg.dynamicSmemBytes = smem_bytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  const bool pdl = p.pdl_wait_all || p.pdl_seg0_wait;
  if (pdl) {  // programmatic dependent of the preceding kernel (see Params::pdl_wait_all / pdl_seg0_wait)
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
  }
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 2 : 1;
  if (cudaLaunchKernelEx(&cfg, kern, w0, t0, w1, t1, p) != cudaSuccess) return DSCA_ERR_CUDA;
  return cudaGetLastError() == cudaSuccess ? DSCA_OK : DSCA_ERR_CUDA;
}

// CTA pairs that can be resident at once (a cluster of two needs two free SMs of one GPC).
static int max_resident_pairs(int num_sms) {
  static volatile int cache[kMaxDevices];  // pairs + 1 per device (0 = not yet queried)
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) dev = -1;
  int cached = dev >= 0 ? __atomic_load_n(&cache[dev], __ATOMIC_ACQUIRE) - 1 : -1;
  if (cached < 0) {
    auto kern = gemm::pair::pair_gemm_kernel<gemm::kEpiSwiGLU, false>;
    constexpr int smem_bytes = gemm::pair::Cfg<gemm::kEpiSwiGLU>::kSmemBytes;
    int n = 0;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes) == cudaSuccess) {
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3((unsigned)(num_sms & ~1));
      cfg.blockDim = dim3(gemm::kThreads);
      cfg.dynamicSmemBytes = smem_bytes;
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeClusterDimension;
      attr[0].val.clusterDim.x = 2;
      attr[0].val.clusterDim.y = 1;
      attr[0].val.clusterDim.z = 1;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess) n = 0;
    }
    cudaGetLastError();
    cached = n > 0 ? std::min(n, num_sms / 2) : num_sms / 2;
    if (dev >= 0) __atomic_store_n(&cache[dev], cached + 1, __ATOMIC_RELEASE);
  }
  return cached;
}

static int launch_pair_one(int epi, const CUtensorMap& w0, const CUtensorMap& t0, const CUtensorMap& w1,
                           const CUtensorMap& t1, const gemm::Params& p, int grid, cudaStream_t stream) {
  switch (epi) {
    case gemm::kEpiSwiGLU: return launch_pair<gemm::kEpiSwiGLU>(w0, t0, w1, t1, p, grid, stream);
    case gemm::kEpiSwiGLU2: return launch_pair<gemm::kEpiSwiGLU2>(w0, t0, w1, t1, p, grid, stream);
    case gemm::kEpiReLU: return launch_pair<gemm::kEpiReLU>(w0, t0, w1, t1, p, grid, stream);
    default: return launch_pair<gemm::kEpiStore>(w0, t0, w1, t1, p, grid, stream);
  }
}

int launch_grouped_ffn_bf16_pair(const dsca_ffn_args* f, int num_sms, cudaStream_t stream) {
  const int want = f->num_ctas > 0 ? f->num_ctas : num_sms;
  const int grid = 2 * std::max(1, std::min(want / 2, max_resident_pairs(num_sms)));
  const int segs = f->segments == 0 ? 3 : f->segments;
  const bool shared = f->shared_rows > 0 && (segs & 2);
  const bool routed = (segs & 1) != 0;
  const int phases = f->phases == 0 ? 3 : f->phases;
  if (!routed && !shared) return DSCA_OK;
  if (f->n1p % 256 != 0 || f->dp % 256 != 0 || (shared && f->shared_n1p % 256 != 0)) return DSCA_ERR_BAD_ARG;

  int rc;
  // ---- GEMM1: h = act(a . w1^T)   (+ hs = act(xs . ws1^T))
  if (phases & 1) {
    CUtensorMap w0, t0, w1, t1;
    const bool glu = f->act == DSCA_ACT_SWIGLU;
    // tile_rows 256 (SwiGLU): 128 channels x <= 256 tokens, gate and up halves per CTA
    // (kEpiSwiGLU2); 512: hybrid tiles on the two-accumulator form
    const bool g2 = glu && f->tile_rows != 512;
    const uint32_t wbox = g2 ? gemm::pair::Cfg<gemm::kEpiSwiGLU2>::kWBox : gemm::pair::Cfg<gemm::kEpiSwiGLU>::kWBox;
    const uint32_t tbox = g2 ? gemm::pair::Cfg<gemm::kEpiSwiGLU2>::kTBox
                             : glu ? gemm::pair::Cfg<gemm::kEpiSwiGLU>::kTBox : gemm::pair::Cfg<gemm::kEpiReLU>::kTBox;
    if ((rc = make_map_bf16(&w0, f->w1, (uint64_t)f->num_experts_w * f->n1p, (uint64_t)f->d, wbox))) return rc;
    if ((rc = make_map_bf16(&t0, f->a, (uint64_t)f->capacity, (uint64_t)f->d, tbox))) return rc;
    if (shared) {
      if ((rc = make_map_bf16(&w1, f->ws1, (uint64_t)f->shared_n1p, (uint64_t)f->d, wbox))) return rc;
      if ((rc = make_map_bf16(&t1, f->xs, (uint64_t)f->shared_rows, (uint64_t)f->d, tbox))) return rc;
    } else {
      w1 = w0;
      t1 = t0;
    }
    gemm::Params p{};
    const int epi = g2 ? gemm::kEpiSwiGLU2 : glu ? gemm::kEpiSwiGLU : gemm::kEpiReLU;
    p.epi = epi;
    p.tile_counter = f->tile_counters;  // GEMM1: [0, 2)
    p.seg1_done = (f->shared_handoff == 2 && shared && g2) ? f->tile_counters + 4 : nullptr;  // [4, 6)
    p.err = f->err;
    p.nseg = shared ? 2 : 1;
    // tile_rows 512 (SwiGLU): whole 256-token blocks as non-swapped tiles, the rest swap-AB
    p.hybrid = (glu && f->tile_rows == 512) ? 1 : 0;
    // equal K (the model width) in both segments; right after the permute (SwiGLU) the
    // shared-expert tiles go first and overlap it (programmatic dependent launch)
    p.pdl_seg0_wait = ((p.hybrid || g2) && f->pdl_after_permute && routed) ? 1 : 0;
    p.seg_first = (p.pdl_seg0_wait && shared) ? 1 : 0;
    // interleaved segments: one round of shared tiles first when the permute is still running
    p.l2_hints = f->cache_hints & 1;
    p.l2_ahead = (f->cache_hints >> 8) & 0xff;
    p.interleave_lead = (shared && routed && (f->tile_order & 1)) ? (p.pdl_seg0_wait ? grid / 2 : 0) : -1;
    gemm::set_weight_major(p, f->tile_order);
    gemm::Segment& s0 = p.seg[0];
    s0.group_offsets = f->group_offsets;
    s0.group_weight = f->group_weight;
    s0.group_order = f->group_order;
    s0.ngroups = routed ? f->num_groups : 0;
    s0.rows = 0;
    // SwiGLU: a tile covers 256 output channels (gate and up rows of them; kEpiSwiGLU2: 128,
    // one packed 256-row block); others 256 rows
    s0.n_tiles = (glu && !g2) ? (f->ip + gemm::BN - 1) / gemm::BN : f->n1p / gemm::BN;
    s0.n_full = glu ? f->ip / 128 : 0;
    s0.b_rows_per_group = f->n1p;
    const int kks1 = g2 ? gemm::pair::Cfg<gemm::kEpiSwiGLU2>::kKS : gemm::BK;  // K elements per stage
    s0.k_blocks = (f->d + kks1 - 1) / kks1;
    s0.c = reinterpret_cast<__nv_bfloat16*>(f->h);
    s0.ldc = f->ip;
    s0.n_store = f->ip;
    s0.capacity = f->capacity;
    if (shared) {
      gemm::Segment& s1 = p.seg[1];
      s1.group_offsets = nullptr;
      s1.group_weight = nullptr;
      s1.ngroups = 1;
      s1.rows = f->shared_rows;
      s1.n_tiles = (glu && !g2) ? (f->shared_ip + gemm::BN - 1) / gemm::BN : f->shared_n1p / gemm::BN;
      s1.n_full = glu ? f->shared_ip / 128 : 0;
      s1.b_rows_per_group = f->shared_n1p;
      s1.k_blocks = (f->d + kks1 - 1) / kks1;
      s1.c = reinterpret_cast<__nv_bfloat16*>(f->hs);
      s1.ldc = f->shared_ip;
      s1.n_store = f->shared_ip;
      s1.capacity = f->shared_rows;
    }
    if ((rc = launch_pair_one(epi, w0, t0, w1, t1, p, grid, stream))) return rc;
  }
  // ---- GEMM2: y = h . w2^T   (+ ys = hs . ws2^T)
  if (phases & 2) {
    CUtensorMap w0, t0, w1, t1;
    constexpr uint32_t wbox = gemm::pair::Cfg<gemm::kEpiStore>::kWBox;
    constexpr uint32_t tbox = gemm::pair::Cfg<gemm::kEpiStore>::kTBox;
    if ((rc = make_map_bf16(&w0, f->w2, (uint64_t)f->num_experts_w * f->dp, (uint64_t)f->ip, wbox))) return rc;
    if ((rc = make_map_bf16(&t0, f->h, (uint64_t)f->capacity, (uint64_t)f->ip, tbox))) return rc;
    if (shared) {
      if ((rc = make_map_bf16(&w1, f->ws2, (uint64_t)f->dp, (uint64_t)f->shared_ip, wbox))) return rc;
      if ((rc = make_map_bf16(&t1, f->hs, (uint64_t)f->shared_rows, (uint64_t)f->shared_ip, tbox))) return rc;
    } else {
      w1 = w0;
      t1 = t0;
    }
    gemm::Params p{};
    p.epi = gemm::kEpiStore;
    p.tile_counter = f->tile_counters != nullptr ? f->tile_counters + 2 : nullptr;  // GEMM2: [2, 4)
    p.err = f->err;
    p.nseg = shared ? 2 : 1;
    // the longer K first; with the fused return (ep_ctx) the routed tiles first, so that their
    // NVLink stores drain while the shared-expert tiles compute
    p.seg_first = (shared && f->shared_ip > f->ip && f->ep_ctx == nullptr) ? 1 : 0;
    p.l2_hints = f->cache_hints & 1;
    p.l2_ahead = (f->cache_hints >> 8) & 0xff;
    p.interleave_lead = (shared && routed && (f->tile_order & 1)) ? 0 : -1;
    gemm::set_weight_major(p, f->tile_order);
    p.ep_signal = routed ? static_cast<ep::Ctx*>(f->ep_ctx) : nullptr;
    p.pdl_wait_all = (f->pdl_after_permute && f->ep_ctx == nullptr) ? 1 : 0;  // right after GEMM1
    p.seg1_flag = (p.pdl_wait_all && f->shared_handoff == 2 && shared) ? f->tile_counters + 5 : nullptr;
    p.hybrid = 0;
    gemm::Segment& s0 = p.seg[0];
    s0.ep = static_cast<const ep::Ctx*>(f->ep_ctx);
    s0.group_offsets = f->group_offsets;
    s0.group_weight = f->group_weight;
    s0.group_order = f->group_order;
    s0.ngroups = routed ? f->num_groups : 0;
    s0.rows = 0;
    s0.n_tiles = f->dp / gemm::BN;
    s0.b_rows_per_group = f->dp;
    constexpr int kks = gemm::pair::Cfg<gemm::kEpiStore>::kKS;  // K elements per stage
    s0.k_blocks = (f->ip + kks - 1) / kks;
    s0.c = reinterpret_cast<__nv_bfloat16*>(f->y);
    s0.ldc = f->d;
    s0.n_store = f->d;
    s0.capacity = f->capacity;
    if (shared) {
      gemm::Segment& s1 = p.seg[1];
      s1.group_offsets = nullptr;
      s1.group_weight = nullptr;
      s1.ngroups = 1;
      s1.rows = f->shared_rows;
      s1.n_tiles = f->dp / gemm::BN;
      s1.b_rows_per_group = f->dp;
      s1.k_blocks = (f->shared_ip + kks - 1) / kks;
      s1.c = reinterpret_cast<__nv_bfloat16*>(f->ys);
      s1.ldc = f->d;
      s1.n_store = f->d;
      s1.capacity = f->shared_rows;
    }
    if ((rc = launch_pair_one(gemm::kEpiStore, w0, t0, w1, t1, p, grid, stream))) return rc;
  }
  return DSCA_OK;
}

}  // namespace dsca

// ------------------------------------------------------------------ fp8 weights, two-term tokens
namespace dsca {

static int launch_pair_f8(int epi, const CUtensorMap& w0, const CUtensorMap& t0, const CUtensorMap& w1,
                          const CUtensorMap& t1, const gemm::Params& p, int grid, cudaStream_t stream) {
  switch (epi) {
    case gemm::kEpiSwiGLU: return launch_pair<gemm::kEpiSwiGLU, true>(w0, t0, w1, t1, p, grid, stream);
    case gemm::kEpiReLU: return launch_pair<gemm::kEpiReLU, true>(w0, t0, w1, t1, p, grid, stream);
    default: return launch_pair<gemm::kEpiStore, true>(w0, t0, w1, t1, p, grid, stream);
  }
}

// GEMM1 (e4m3 weights x two-term tokens) -> h, hs in bf16 -> split into hq, hsq -> GEMM2.
int launch_grouped_ffn_f8_split(const dsca_ffn_args* f, int num_sms, cudaStream_t stream) {
  const int want = f->num_ctas > 0 ? f->num_ctas : num_sms;
  const int grid = 2 * std::max(1, std::min(want / 2, max_resident_pairs(num_sms)));
  const int segs = f->segments == 0 ? 3 : f->segments;
  const bool shared = f->shared_rows > 0 && (segs & 2);
  const bool routed = (segs & 1) != 0;
  const int phases = f->phases == 0 ? 3 : f->phases;
  if (!routed && !shared) return DSCA_OK;
  if (f->ep_ctx != nullptr) return DSCA_ERR_UNSUPPORTED;
  if (f->n1p % 256 != 0 || f->dp % 256 != 0 || (shared && f->shared_n1p % 256 != 0)) return DSCA_ERR_BAD_ARG;
  if (f->ip % 128 != 0 || (shared && f->shared_ip % 128 != 0) || f->d % 16 != 0) return DSCA_ERR_BAD_ARG;
  const bool glu = f->act == DSCA_ACT_SWIGLU;
  const int Kd = (f->d + 127) & ~127;  // token row: [hi: Kd | lo: Kd] bytes
  int rc;
  if ((phases & 1) && f->tile_rows != 256) {
    // GEMM1 on single-CTA tiles (as the bf16 default), then the intermediates' split below
    if ((rc = launch_gemm1_f8_single(f, num_sms, stream))) return rc;
  } else if (phases & 1) {
    using CG = gemm::pair::Cfg<gemm::kEpiSwiGLU, true>;
    using CR = gemm::pair::Cfg<gemm::kEpiReLU, true>;
    const uint32_t tbox = glu ? CG::kTBox : CR::kTBox;
    CUtensorMap w0, t0, w1, t1;
    if ((rc = make_map_e4m3(&w0, f->w1, (uint64_t)f->num_experts_w * f->n1p, (uint64_t)f->d, CG::kWBox))) return rc;
    if ((rc = make_map_e4m3(&t0, f->a, (uint64_t)std::max(f->capacity, 1), (uint64_t)2 * Kd, tbox))) return rc;
    if (shared) {
      if ((rc = make_map_e4m3(&w1, f->ws1, (uint64_t)f->shared_n1p, (uint64_t)f->d, CG::kWBox))) return rc;
      if ((rc = make_map_e4m3(&t1, f->xs, (uint64_t)f->shared_rows, (uint64_t)2 * Kd, tbox))) return rc;
    } else {
      w1 = w0;
      t1 = t0;
    }
    gemm::Params p{};
    const int epi = glu ? gemm::kEpiSwiGLU : gemm::kEpiReLU;
    p.epi = epi;
    p.tile_counter = f->tile_counters;  // GEMM1: [0, 2)
    p.err = f->err;
    p.nseg = shared ? 2 : 1;
    p.seg_first = 0;
    p.interleave_lead = -1;
    gemm::set_weight_major(p, f->tile_order);
    p.l2_hints = f->cache_hints & 1;
    p.l2_ahead = (f->cache_hints >> 8) & 0xff;
    gemm::Segment& s0 = p.seg[0];
    s0.group_offsets = f->group_offsets;
    s0.group_weight = f->group_weight;
    s0.group_order = f->group_order;
    s0.ngroups = routed ? f->num_groups : 0;
    s0.n_tiles = glu ? (f->ip + gemm::BN - 1) / gemm::BN : f->n1p / gemm::BN;
    s0.b_rows_per_group = f->n1p;
    s0.k_blocks = (f->d + 127) / 128;
    s0.c = reinterpret_cast<__nv_bfloat16*>(f->h);
    s0.ldc = f->ip;
    s0.n_store = f->ip;
    s0.capacity = f->capacity;
    s0.t_lo = Kd;
    s0.t_scale = f->a_scale;
    s0.w_scale = f->w1_scale;
    if (shared) {
      gemm::Segment& s1 = p.seg[1];
      s1.ngroups = 1;
      s1.rows = f->shared_rows;
      s1.n_tiles = glu ? (f->shared_ip + gemm::BN - 1) / gemm::BN : f->shared_n1p / gemm::BN;
      s1.b_rows_per_group = f->shared_n1p;
      s1.k_blocks = (f->d + 127) / 128;
      s1.c = reinterpret_cast<__nv_bfloat16*>(f->hs);
      s1.ldc = f->shared_ip;
      s1.n_store = f->shared_ip;
      s1.capacity = f->shared_rows;
      s1.t_lo = Kd;
      s1.t_scale = f->xs_scale;
      s1.w_scale = f->ws1_scale;
    }
    if ((rc = launch_pair_f8(epi, w0, t0, w1, t1, p, grid, stream))) return rc;
  }
  if (phases & 1) {
    // the intermediates as two-term rows for GEMM2 (routed rows: as many as the groups hold)
    if (routed && (rc = launch_split_rows(f->h, f->ip, f->capacity, f->group_offsets + f->num_groups, f->ip, f->hq,
                                          f->h_scale, stream)))
      return rc;
    if (shared && (rc = launch_split_rows(f->hs, f->shared_ip, f->shared_rows, nullptr, f->shared_ip, f->hsq,
                                          f->hs_scale, stream)))
      return rc;
  }
  if (phases & 2) {
    using CS = gemm::pair::Cfg<gemm::kEpiStore, true>;
    CUtensorMap w0, t0, w1, t1;
    if ((rc = make_map_e4m3(&w0, f->w2, (uint64_t)f->num_experts_w * f->dp, (uint64_t)f->ip, CS::kWBox))) return rc;
    if ((rc = make_map_e4m3(&t0, f->hq, (uint64_t)std::max(f->capacity, 1), (uint64_t)2 * f->ip, CS::kTBox)))
      return rc;
    if (shared) {
      if ((rc = make_map_e4m3(&w1, f->ws2, (uint64_t)f->dp, (uint64_t)f->shared_ip, CS::kWBox))) return rc;
      if ((rc = make_map_e4m3(&t1, f->hsq, (uint64_t)f->shared_rows, (uint64_t)2 * f->shared_ip, CS::kTBox)))
        return rc;
    } else {
      w1 = w0;
      t1 = t0;
    }
    gemm::Params p{};
    p.epi = gemm::kEpiStore;
    p.tile_counter = f->tile_counters != nullptr ? f->tile_counters + 2 : nullptr;  // GEMM2: [2, 4)
    p.err = f->err;
    p.nseg = shared ? 2 : 1;
    p.seg_first = (shared && f->shared_ip > f->ip) ? 1 : 0;  // the longer K first
    p.interleave_lead = -1;
    gemm::set_weight_major(p, f->tile_order);
    p.l2_hints = f->cache_hints & 1;
    p.l2_ahead = (f->cache_hints >> 8) & 0xff;
    gemm::Segment& s0 = p.seg[0];
    s0.group_offsets = f->group_offsets;
    s0.group_weight = f->group_weight;
    s0.group_order = f->group_order;
    s0.ngroups = routed ? f->num_groups : 0;
    s0.n_tiles = f->dp / gemm::BN;
    s0.b_rows_per_group = f->dp;
    s0.k_blocks = f->ip / 128;
    s0.c = reinterpret_cast<__nv_bfloat16*>(f->y);
    s0.ldc = f->d;
    s0.n_store = f->d;
    s0.capacity = f->capacity;
    s0.t_lo = f->ip;
    s0.t_scale = f->h_scale;
    s0.w_scale = f->w2_scale;
    if (shared) {
      gemm::Segment& s1 = p.seg[1];
      s1.ngroups = 1;
      s1.rows = f->shared_rows;
      s1.n_tiles = f->dp / gemm::BN;
      s1.b_rows_per_group = f->dp;
      s1.k_blocks = f->shared_ip / 128;
      s1.c = reinterpret_cast<__nv_bfloat16*>(f->ys);
      s1.ldc = f->d;
      s1.n_store = f->d;
      s1.capacity = f->shared_rows;
      s1.t_lo = f->shared_ip;
      s1.t_scale = f->hs_scale;
      s1.w_scale = f->ws2_scale;
    }
    if ((rc = launch_pair_f8(gemm::kEpiStore, w0, t0, w1, t1, p, grid, stream))) return rc;
  }
  return DSCA_OK;
}

}  // namespace dsca
